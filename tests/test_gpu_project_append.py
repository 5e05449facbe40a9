"""Fused latent projection + quantise-append (``starkv_project_append``).

Two copies of a prefilled cache: one gets the decode token through the fused
entry point (which also returns its rounded latents), the other through the
existing ``starkv_append`` fed those latents.  Codes, scales/zeros (or the
unquantised rows) must be bit-identical, and the latents must match the fp32
projection ``hidden @ VS^T`` rounded to the latent dtype (accumulation order
differs: rel-L2 <= 1e-3)."""

import numpy as np
import pytest
import torch

from starkv import ops
from starkv.harness import build_step
from starkv.synthetic import make_layer, make_spec

pytestmark = pytest.mark.gpu


def _clone(cache):
    c = ops.LatentCache(cache.layout, device=cache.k_cache.device)
    for name in ("k_cache", "k_scales", "v_cache", "v_params"):
        t = getattr(cache, name)
        if t is not None:
            getattr(c, name).copy_(t)
    c.length = cache.length
    return c


@pytest.mark.parametrize("cfg,over,H", [
    ("c1", dict(num_q_heads=8, batch=3, context=50), 512),
    ("c1", dict(num_q_heads=32, batch=11, context=20), 4096),          # two batch passes of 8
    ("c0", dict(num_q_heads=8, batch=2, context=40), 256),
    ("c0", dict(num_q_heads=8, batch=2, context=40, dtype="bfloat16"), 256),
    ("c2", dict(num_q_heads=32, num_kv_heads=8, batch=2, context=30), 1024),
])
def test_project_append_matches_append(cuda, cfg, over, H):
    spec = make_spec(cfg, seed=21, **over)
    st = build_step(make_layer(spec), cuda)
    base = st.layer.cache
    dt = base.latent_dtype
    L = base.layout
    g = torch.Generator(device=cuda).manual_seed(4)
    hidden = torch.randn(L.batch, 1, H, generator=g, device=cuda).to(dt)
    vs_k = (torch.randn(L.k_rank_total, H, generator=g, device=cuda) / H ** 0.5).to(dt)
    vs_v = (torch.randn(L.v_rank_total, H, generator=g, device=cuda) / H ** 0.5).to(dt)
    fused, ref = _clone(base), _clone(base)
    k_lat, v_lat = fused.project_append(hidden, vs_k, vs_v, return_latents=True)
    ref.append(k_lat, v_lat)
    torch.cuda.synchronize()
    assert fused.length == ref.length == base.length + 1
    for name in ("k_cache", "k_scales", "v_cache", "v_params"):
        a, b = getattr(fused, name), getattr(ref, name)
        if a is not None:
            assert torch.equal(a, b), name
    for lat, vs in ((k_lat, vs_k), (v_lat, vs_v)):
        want = (hidden.float().reshape(L.batch, H) @ vs.float().T).to(dt).float().cpu().numpy()
        got = lat.float().reshape(L.batch, -1).cpu().numpy()
        assert np.linalg.norm(got - want) / np.linalg.norm(want) <= 1e-3


@pytest.mark.parametrize("batch", [4, 12])
def test_step_from_hidden_routes_by_batch(cuda, batch):
    """``DecodeLayer.step_from_hidden`` uses the fused projection up to 8 sequences and
    two cuBLAS GEMMs + ``starkv_append`` above; both give the attention of
    ``append(hidden @ VS^T)`` (the latents may differ in the last bit: GEMM
    accumulation order), within the decode tolerance."""
    spec = make_spec("c1", seed=22, num_q_heads=8, batch=batch, context=300)
    st = build_step(make_layer(spec), cuda)
    L = st.layer
    H = 512
    g = torch.Generator(device=cuda).manual_seed(5)
    dt = L.cache.latent_dtype
    hidden = torch.randn(batch, 1, H, generator=g, device=cuda).to(dt)
    vs_k = (torch.randn(L.layout.k_rank_total, H, generator=g, device=cuda) / H ** 0.5).to(dt)
    vs_v = (torch.randn(L.layout.v_rank_total, H, generator=g, device=cuda) / H ** 0.5).to(dt)
    ref_cache = _clone(L.cache)
    out = torch.empty(batch, spec.num_q_heads, 128, dtype=torch.float32, device=cuda)
    L.step_from_hidden(st.q, hidden, vs_k, vs_v, out=out)
    k_lat = (hidden.float() @ vs_k.float().T).to(dt)
    v_lat = (hidden.float() @ vs_v.float().T).to(dt)
    ref_cache.append(k_lat.contiguous(), v_lat.contiguous())
    want = ops.decode_attention(L.layout, ref_cache, st.q, L.k_u, L.v_u, L.inv_freq, L.scaling,
                                ref_cache.length).float().cpu().numpy()
    got = out.cpu().numpy()
    assert np.linalg.norm(got - want) / np.linalg.norm(want) <= 2e-3
