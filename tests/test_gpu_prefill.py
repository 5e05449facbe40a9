"""Prompt (prefill) attention on the B200 through the C ABI
(``starkv_prefill_attention``) against the CPU oracle's restatement of the
reference's prefill (model.py:429-449) and against plain fp32 causal attention.

Tolerance (north star): rel-L2 <= 2e-3 and max-abs <= 1e-2 against the fp32/fp64
reference for fp16 inputs.  bf16 inputs round the softmax weights to bf16 before
P.V (as any bf16 flash attention does), so there the error is bounded by twice
that of torch's own bf16 SDPA against the same fp32 reference."""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import starkv_oracle as O
from starkv import ops, prefill
from starkv.layer import rope_inv_freq
from starkv.synthetic import make_layer, make_spec

pytestmark = pytest.mark.gpu
REL_L2, MAX_ABS = 2e-3, 1e-2


def _ref_f32(q, k, v, scaling):
    """Causal attention in fp32 with the K / V heads repeated for GQA."""
    grp = q.shape[1] // k.shape[1]
    k = k.float().repeat_interleave(grp, dim=1)
    v = v.float().repeat_interleave(grp, dim=1)
    s = torch.matmul(q.float(), k.transpose(-1, -2)) * scaling
    T = q.shape[2]
    s = s.masked_fill(~torch.ones(T, T, dtype=torch.bool, device=q.device).tril(), float("-inf"))
    return torch.matmul(torch.softmax(s, dim=-1), v)


def _rel(a, b):
    return (torch.linalg.vector_norm((a - b).double()) / torch.linalg.vector_norm(b.double())).item()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("B,Hq,Hkv,T", [(2, 8, 2, 300), (1, 4, 4, 128), (1, 2, 1, 1), (1, 2, 2, 129),
                                        (3, 6, 3, 517), (1, 2, 1, 16384)])
def test_prefill_kernel_matches_fp32_attention(cuda, dtype, B, Hq, Hkv, T):
    g = torch.Generator(device=cuda).manual_seed(B * 1000 + T)
    # (B, T, H, 128) projections read through transposed views, as the module passes them
    q = torch.randn(B, T, Hq, 128, generator=g, device=cuda).to(dtype).transpose(1, 2)
    k = torch.randn(B, T, Hkv, 128, generator=g, device=cuda).to(dtype).transpose(1, 2)
    v = torch.randn(B, T, Hkv, 128, generator=g, device=cuda).to(dtype).transpose(1, 2)
    scaling = 128 ** -0.5
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = ops.prefill_attention(q, k, v, scaling, out_dtype=torch.float32, error_word=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = _ref_f32(q, k, v, scaling)
    rel, mx = _rel(out, ref), (out - ref).abs().max().item()
    if dtype == torch.float16:
        assert rel <= REL_L2 and mx <= MAX_ABS, (rel, mx)
    else:
        grp = Hq // Hkv
        sdpa = F.scaled_dot_product_attention(q, k.repeat_interleave(grp, 1), v.repeat_interleave(grp, 1),
                                              is_causal=True, scale=scaling).float()
        assert rel <= max(2 * _rel(sdpa, ref), REL_L2), (rel, _rel(sdpa, ref))
    # model-dtype output is the fp32 result rounded
    o16 = ops.prefill_attention(q, k, v, scaling)
    assert o16.dtype == dtype
    assert torch.equal(o16, out.to(dtype))


def test_prefill_rejects_bad_arguments(cuda):
    q = torch.zeros(1, 4, 16, 128, dtype=torch.float16, device=cuda)
    kv = torch.zeros(1, 3, 16, 128, dtype=torch.float16, device=cuda)
    with pytest.raises(Exception):
        ops.prefill_attention(q, kv, kv, 1.0)                       # 4 query heads over 3 KV heads
    with pytest.raises(Exception):
        ops.prefill_attention(q.float(), q.float(), q.float(), 1.0)  # fp32 inputs


@pytest.mark.parametrize("cfg,over", [("c2", dict(num_q_heads=8, num_kv_heads=2, batch=1, context=2047)),
                                      ("c1", dict(num_q_heads=4, batch=1, context=1500))])
def test_prompt_path_matches_oracle(cuda, cfg, over):
    """A 2K-token prompt through the latent rebuild + tcgen05 attention against the
    oracle's restatement of the reference prefill (float64)."""
    spec = make_spec(cfg, seed=21, quantized=False, **over)
    data = make_layer(spec)
    T = spec.context + 1
    dt = getattr(torch, spec.dtype)
    rng = np.random.default_rng(5)
    q = rng.standard_normal((spec.batch, spec.num_q_heads, T, 128)).astype(np.float32)
    q16 = torch.from_numpy(q).to(cuda, dt)
    k_lat = torch.from_numpy(np.concatenate(data.xk, axis=-1)).to(cuda, dt)
    v_lat = torch.from_numpy(data.xv).to(cuda, dt)
    k_u = [torch.from_numpy(u).to(cuda, dt) for u in data.k_u]
    v_u = torch.from_numpy(data.v_u).to(cuda, dt)
    inv = rope_inv_freq(spec.theta, 128, cuda)
    ang = torch.arange(T, device=cuda, dtype=torch.float32)[:, None] * inv[None]
    emb = torch.cat([ang, ang], dim=-1)[None]
    cos, sin = emb.cos().to(dt), emb.sin().to(dt)
    keys = prefill.rebuild_keys(k_lat, k_u, spec.k_ranks, cos, sin)
    vals = prefill.rebuild_values(v_lat, v_u, spec.num_kv_heads)
    scaling = 128 ** -0.5
    out = prefill.prompt_attention(q16, keys, vals, scaling, out_dtype=torch.float32)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    # the oracle sees the same 16-bit inputs (the GPU path rounds them once on upload)
    q_in = q16.float().cpu().numpy()
    xk = [x.astype(np.float32) for x in data.xk]
    xk = [torch.from_numpy(x).to(dt).float().numpy() for x in xk]
    xv = torch.from_numpy(data.xv).to(dt).float().numpy()
    ku = [torch.from_numpy(u).to(dt).float().numpy() for u in data.k_u]
    vu = torch.from_numpy(data.v_u).to(dt).float().numpy()
    blk = spec.v_block_of_kv()
    ref = O.prompt_attention(q_in, xk, ku, xv, vu, spec.k_ranks, spec.v_ranks, blk,
                             inv.cpu().numpy(), scaling)
    rel, mx = O.rel_l2(got, ref), float(np.abs(got - ref).max())
    # K / V are rebuilt in the model dtype before attention (as the reference's
    # matmuls do), which bounds the agreement for bf16 layers
    tol = REL_L2 if dt == torch.float16 else 1e-2
    assert rel <= tol and mx <= (MAX_ABS if dt == torch.float16 else 5e-2), (rel, mx)
