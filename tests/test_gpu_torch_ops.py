"""torch.ops.starkv.* on the GPU give the same results as the ctypes wrappers."""

import numpy as np
import pytest
import torch

from starkv import ops, torch_ops
from starkv.harness import build_step
from starkv.synthetic import make_layer, make_spec

pytestmark = pytest.mark.gpu


def test_torch_ops_match_the_wrappers(cuda):
    spec = make_spec("c1", seed=41, num_q_heads=8, batch=2, context=700)
    st = build_step(make_layer(spec), cuda)
    L = st.layer
    c = L.cache
    lt = torch_ops.layout_tensor(L.layout)
    T = L.length
    torch.ops.starkv.quant_append(lt, st.k_new, st.v_new, T, c.k_cache, c.k_scales, c.v_cache, c.v_params)
    c.length = T + 1
    T += 1
    want = ops.decode_attention(L.layout, c, st.q, L.k_u, L.v_u, L.inv_freq, L.scaling, T)
    got = torch.ops.starkv.decode_attn(lt, st.q, L.k_u, L.v_u, L.inv_freq, c.k_cache, c.k_scales, c.v_cache,
                                       c.v_params, L.scaling, T)
    assert torch.equal(got, want)
    lg = torch.ops.starkv.k_attn(lt, st.q, L.k_u, L.inv_freq, c.k_cache, c.k_scales, T)
    assert torch.equal(lg, ops.k_logits(L.layout, c, st.q, L.k_u, L.inv_freq, T))
    p = torch.softmax(lg * L.scaling, dim=-1).contiguous()
    v = torch.ops.starkv.v_attn(lt, p, c.v_cache, c.v_params, T)
    assert torch.equal(v, ops.v_latent(L.layout, c, p, T))
    assert np.isfinite(got.float().cpu().numpy()).all()
