"""Quantise / append kernels: bit-exact against the CPU oracle (through the C ABI)."""

import numpy as np
import pytest
import torch

import starkv_oracle as O
from starkv import ops
from starkv.harness import build_step
from starkv.synthetic import make_layer, make_spec

pytestmark = pytest.mark.gpu


def _np16(t):
    return t.cpu().numpy()


@pytest.mark.parametrize("cfg,over", [
    ("c1", dict(num_q_heads=8, batch=2, context=515)),
    ("c1", dict(num_q_heads=4, batch=3, context=1)),
    ("c2", dict(num_q_heads=16, num_kv_heads=4, batch=2, context=640)),
    ("c1", dict(num_q_heads=8, batch=1, context=300, dtype="float32")),
])
def test_prefill_and_append_bit_exact(cuda, cfg, over):
    spec = make_spec(cfg, seed=3, **over)
    data = make_layer(spec)
    st = build_step(data, cuda)
    st.layer.append(st.k_new, st.v_new)
    torch.cuda.synchronize()
    ref = O.quantize_layer(data.xk, data.xv, spec.context)
    cache = st.layer.cache
    lay = st.layer.layout
    T = spec.tokens
    ks = _np16(cache.k_scales).reshape(spec.batch, -1)
    for h in range(spec.num_kv_heads):
        c0 = lay.k_col[h]
        np.testing.assert_array_equal(ks[:, c0:c0 + spec.k_ranks[h]], ref["k_scales"][h])
        np.testing.assert_array_equal(cache.k_head(h)[:, :T].cpu().numpy(), ref["k_codes"][h])
    np.testing.assert_array_equal(cache.v_cache[:, :T].cpu().numpy(), ref["v_codes"])
    vp = cache.v_params[:, :T].cpu().numpy()
    np.testing.assert_array_equal(vp[..., 0], ref["v_scale"])
    np.testing.assert_array_equal(vp[..., 1], ref["v_zero"])


def test_append_saturates_and_handles_constant_groups(cuda):
    spec = make_spec("c1", seed=5, num_q_heads=4, batch=2, context=64)
    data = make_layer(spec)
    data.xk[0][:, -1, :] = (data.xk[0][:, -1, :] * 50.0).astype(np.float16).astype(np.float32)  # beyond the prefill range
    data.xv[:, -1, :32] = 0.25                       # constant group
    st = build_step(data, cuda)
    st.layer.append(st.k_new, st.v_new)
    ref = O.quantize_layer(data.xk, data.xv, spec.context)
    np.testing.assert_array_equal(st.layer.cache.k_head(0)[:, :spec.tokens].cpu().numpy(), ref["k_codes"][0])
    np.testing.assert_array_equal(st.layer.cache.v_cache[:, :spec.tokens].cpu().numpy(), ref["v_codes"])
    assert np.abs(ref["k_codes"][0][:, -1]).max() == 127


def test_append_rejects_overflow(cuda):
    spec = make_spec("c1", seed=5, num_q_heads=4, batch=1, context=10)
    st = build_step(make_layer(spec), cuda)
    st.layer.cache.length = st.layer.layout.capacity - 1   # capacity: tokens rounded up to a 128-slot tile
    st.layer.append(st.k_new, st.v_new)                    # fills the last slot
    with pytest.raises(ops._lib.StarKVError):
        st.layer.append(st.k_new, st.v_new)
