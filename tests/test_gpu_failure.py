"""Device-side failure path of the K kernel, made without faulting the GPU.

A test hook shortens every device wait to 20 ms and makes the first CTA's
producer never issue one unit's staging copy.  The waits on that stage run
out; the kernel records an error code in the workspace's first word, its roles
leave their loops, wait (bounded) for their copies and MMAs in flight, free
TMEM and return.  The host reads the code, and the next normal step on the same
device still matches the oracle."""

import numpy as np
import pytest

import starkv_oracle as O
from starkv import ops
from starkv.harness import build_step
from starkv.synthetic import make_layer, make_spec

pytestmark = pytest.mark.gpu
REL_L2, MAX_ABS = 2e-3, 1e-2
DEV_WAIT_COPY, DEV_WAIT_MMA = 0x101, 0x102


def test_timed_out_wait_reports_and_the_device_recovers(cuda):
    spec = make_spec("c1", seed=31, num_q_heads=8, batch=2, context=3000)
    data = make_layer(spec)
    st = build_step(data, cuda)
    L = st.layer
    L.append(st.k_new, st.v_new)
    assert ops.read_device_error(device=cuda) == 0
    try:
        ops.set_test_hooks(wait_limit_ns=20_000_000, skip_copy_unit=1)
        L.attend(st.q)
        code = ops.read_device_error(device=cuda)
    finally:
        ops.set_test_hooks()
    assert code in (DEV_WAIT_COPY, DEV_WAIT_MMA), hex(code)
    out = L.attend(st.q, out=None).float().cpu().numpy()
    assert ops.read_device_error(device=cuda) == 0
    ref = O.layer_reference(data)
    assert O.rel_l2(out, ref) <= 1e-2           # model-dtype output (fp16)
    assert np.abs(out - ref).max() <= 2e-2
