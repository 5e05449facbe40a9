"""The decode step for callers that cannot allocate device memory while they run
it (plugins handed only input/output buffers, code under another framework's
memory pool): ``starkv_decode_attention_static`` uses the library's fixed static
scratch instead of a caller workspace.  Checked through the C ABI against the
ordinary entry point, twice in a row (the scratch keeps the previous call's
contents), and for its size limit.  Collected last on purpose."""

import ctypes as C

import numpy as np
import pytest
import torch

import starkv_oracle as O
from starkv import _lib, ops
from starkv.harness import build_step, device_layer
from starkv.synthetic import make_layer, make_spec

pytestmark = pytest.mark.gpu
REL_L2, MAX_ABS = 2e-3, 1e-2


def test_static_scratch_matches_workspace_entry_point(cuda):
    spec = make_spec("c1", seed=21, num_q_heads=8, batch=2, context=2500)
    st = build_step(make_layer(spec), cuda)
    layer = st.layer
    layer.append(st.k_new, st.v_new)
    T = layer.length
    ref = ops.decode_attention(layer.layout, layer.cache, st.q, layer.k_u, layer.v_u, layer.inv_freq,
                               layer.scaling, T).float().cpu().numpy()
    for _ in range(2):
        out = torch.full_like(st.q, float("nan"))
        ops.decode_attention_static(layer.layout, layer.cache, st.q, layer.k_u, layer.v_u, layer.inv_freq,
                                    layer.scaling, T, out)
        torch.cuda.synchronize()
        got = out.float().cpu().numpy()
        assert ops.static_read_device_error() == 0
        assert np.isfinite(got).all()
        assert O.rel_l2(got, ref) <= REL_L2
        assert np.abs(got - ref).max() <= MAX_ABS


def test_static_scratch_near_its_limit(cuda):
    """A step whose scratch fills the static array to within a few KB: the last
    regions of the scratch (256-byte aligned offsets near the end) are used."""
    lib = _lib.load()
    cap = lib.starkv_static_scratch_bytes()
    spec = make_spec("c1", seed=23, num_q_heads=32, batch=16, context=1000)
    lay = ops.layout_from_spec(spec)
    lo, hi = 1000, 32768                                        # largest context whose step still fits
    while lo < hi:
        mid = (lo + hi + 1) // 2
        if ops.workspace_size(lay, mid + 1) <= cap:
            lo = mid
        else:
            hi = mid - 1
    spec.context = lo
    assert cap - ops.workspace_size(ops.layout_from_spec(spec), spec.tokens) < 64 * 1024
    st, _, _ = device_layer(spec, cuda, seed=3)
    layer = st.layer
    layer.append(st.k_new, st.v_new)
    T = layer.length
    ref = ops.decode_attention(layer.layout, layer.cache, st.q, layer.k_u, layer.v_u, layer.inv_freq,
                               layer.scaling, T).float().cpu().numpy()
    out = torch.full_like(st.q, float("nan"))
    ops.decode_attention_static(layer.layout, layer.cache, st.q, layer.k_u, layer.v_u, layer.inv_freq,
                                layer.scaling, T, out)
    got = out.float().cpu().numpy()
    assert ops.static_read_device_error() == 0
    assert O.rel_l2(got, ref) <= REL_L2
    assert np.abs(got - ref).max() <= MAX_ABS


def test_static_scratch_rejects_oversized_steps(cuda):
    lib = _lib.load()
    cap = lib.starkv_static_scratch_bytes()
    spec = make_spec("c1", seed=22, num_q_heads=32, batch=16, context=32768)
    lay = ops.layout_from_spec(spec)
    assert ops.workspace_size(lay, spec.tokens) > cap
    a = _lib.DecodeArgs()
    a.num_tokens = spec.tokens
    rc = lib.starkv_decode_attention_static(C.byref(lay), C.byref(a), None)
    assert rc == 4                                              # STARKV_ERR_WORKSPACE
    assert b"static scratch" in lib.starkv_last_error()
