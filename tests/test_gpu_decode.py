"""Decode attention on the B200 against the reference (golden vectors made by the
reference's own eager module) and the CPU oracle, through the C ABI.

Tolerance (north star): rel-L2 <= 2e-3 and max-abs <= 1e-2 against the fp32 reference."""

import json
import os

import numpy as np
import pytest
import torch

import starkv_oracle as O
from starkv import ops
from starkv.harness import build_step, device_layer
from starkv.synthetic import make_layer, make_spec

from conftest import GOLDEN

pytestmark = pytest.mark.gpu
REL_L2, MAX_ABS = 2e-3, 1e-2
MANIFEST = json.load(open(os.path.join(GOLDEN, "manifest.json")))


def _run(data, cuda, num_splits=0):
    """One decode step; the attention output is requested in fp32 so the tolerance
    measures the computation (the model-dtype output is that result rounded,
    checked in test_model_dtype_output_is_rounded_fp32)."""
    st = build_step(data, cuda)
    st.layer.append(st.k_new, st.v_new)
    L = st.layer
    out = torch.empty(data.spec.batch, data.spec.num_q_heads, 128, dtype=torch.float32, device=cuda)
    ops.decode_attention(L.layout, L.cache, st.q, L.k_u, L.v_u, L.inv_freq, L.scaling, L.length,
                         mask=st.mask, out=out, num_splits=num_splits)
    torch.cuda.synchronize()
    assert ops.read_device_error(device=cuda) == 0
    return out.cpu().numpy(), st


@pytest.mark.parametrize("cfg,over", [("c1", dict(num_q_heads=8, batch=2, context=1000)),
                                      ("c2", dict(num_q_heads=16, num_kv_heads=4, batch=2, context=1000))])
def test_model_dtype_output_is_rounded_fp32(cuda, cfg, over):
    spec = make_spec(cfg, seed=15, **over)
    data = make_layer(spec)
    f32, st = _run(data, cuda)
    L = st.layer
    out = ops.decode_attention(L.layout, L.cache, st.q, L.k_u, L.v_u, L.inv_freq, L.scaling, L.length)
    assert out.dtype == st.q.dtype
    rounded = torch.from_numpy(f32).to(out.dtype).float().numpy()
    got = out.float().cpu().numpy()
    eps = 2.0 ** (-8 if out.dtype == torch.bfloat16 else -11)
    assert np.all(np.abs(got - rounded) <= eps * np.abs(rounded) + 1e-6)


@pytest.mark.parametrize("name", sorted(MANIFEST))
def test_decode_matches_reference_golden(cuda, name):
    m = MANIFEST[name]
    spec = make_spec(m["config"], seed=0, **m["overrides"])
    data = make_layer(spec, with_mask=m["with_mask"])
    out, _ = _run(data, cuda)
    gold = np.load(os.path.join(GOLDEN, f"{name}.npz"))["attn"].reshape(out.shape)
    assert O.rel_l2(out, gold) <= REL_L2
    assert np.abs(out - gold).max() <= MAX_ABS


@pytest.mark.parametrize("cfg,over,mask", [
    ("c1", dict(num_q_heads=8, batch=2, context=127), False),     # T = 128 exactly
    ("c1", dict(num_q_heads=8, batch=2, context=128), False),     # T = 129 (one-row tail)
    ("c1", dict(num_q_heads=4, batch=1, context=1), False),       # T = 2
    ("c1", dict(num_q_heads=12, batch=2, context=900), False),    # 12 heads: a partial group of 8 in the V prob warps
    ("c1", dict(num_q_heads=32, batch=3, context=1500), True),
    ("c2", dict(num_q_heads=32, num_kv_heads=8, batch=2, context=2000), False),
    ("c0", dict(num_q_heads=8, batch=2, context=700, dtype="float16"), False),
    ("c0", dict(num_q_heads=8, batch=2, context=700, dtype="bfloat16"), True),
    # V blocks with more than 8 query heads and ranks above one 256-channel CTA tile
    ("c0", dict(num_q_heads=32, batch=1, context=300, v_block_kv=[16, 16], v_ranks=[512, 320]), False),
    ("c1", dict(num_q_heads=32, batch=2, context=600, v_block_kv=[32], v_ranks=[1024]), False),
])
def test_decode_matches_oracle(cuda, cfg, over, mask):
    spec = make_spec(cfg, seed=11, **over)
    data = make_layer(spec, with_mask=mask)
    out, _ = _run(data, cuda)
    ref = O.layer_reference(data)
    assert O.rel_l2(out, ref) <= REL_L2
    assert np.abs(out - ref).max() <= MAX_ABS


@pytest.mark.parametrize("ranks,context,batch", [
    ([96], 40, 2),           # one M unit, one tile: five of six accumulator replicas stay empty
    ([96], 3000, 2),         # one M unit, six replicas
    ([96], 8000, 16),        # ... with ~14 tiles per V split: every B tile buffer reused
    ([128, 64], 2000, 2),    # two units, three replicas each
    ([128, 64], 6000, 16),
    ([192, 192], 1500, 2),   # three units, two replicas
    ([192, 192], 6000, 16),
    ([256, 256], 1500, 2),   # four units, one replica
    ([320, 320], 900, 2),    # five units
    # seven, ten and thirteen units: the units past the last multiple of six rotate
    # over the pairs tile by tile (rotating tail), each pair with its own accumulator
    ([256, 256, 256, 64], 1500, 2),
    ([256, 256, 256, 64], 6000, 16),
    ([256, 256, 256, 256, 128, 96], 3000, 4),
    ([256, 256, 256, 256, 256, 256, 64], 2000, 4),
])
def test_v_units_and_replicas(cuda, ranks, context, batch):
    """V layers whose 128-channel units do not fill six dequant warp pairs evenly:
    fewer than six units (head shards) split the tiles into per-replica
    accumulators; past a multiple of six the tail units rotate over the pairs."""
    nb = len(ranks)
    blocks = [8 // nb + (1 if j < 8 % nb else 0) for j in range(nb)]
    spec = make_spec("c1", seed=16, num_q_heads=8, batch=batch, context=context,
                     v_block_kv=blocks, v_ranks=ranks)
    data = make_layer(spec)
    ref = O.layer_reference(data)
    for ns in (0, 1, 5):
        out, _ = _run(data, cuda, num_splits=ns)
        assert O.rel_l2(out, ref) <= REL_L2
        assert np.abs(out - ref).max() <= MAX_ABS


def test_split_count_invariance_and_determinism(cuda):
    spec = make_spec("c1", seed=12, num_q_heads=8, batch=2, context=3000)
    data = make_layer(spec)
    a, _ = _run(data, cuda, num_splits=1)
    b, _ = _run(data, cuda, num_splits=7)
    c, _ = _run(data, cuda, num_splits=7)
    np.testing.assert_array_equal(b, c)
    assert O.rel_l2(a, b) < 2e-4            # outputs are fp16: split order only moves the last bit


def test_k_logits_matches_oracle(cuda):
    """abx's contract: unscaled q . RoPE(X U^T) per position."""
    spec = make_spec("c1", seed=13, num_q_heads=8, batch=2, context=900)
    data = make_layer(spec)
    st = build_step(data, cuda)
    st.layer.append(st.k_new, st.v_new)
    T = spec.tokens
    lg = ops.k_logits(st.layer.layout, st.layer.cache, st.q, st.layer.k_u, st.layer.inv_freq, T)
    qz = O.quantize_layer(data.xk, data.xv, spec.context)
    cos, sin = O.rope_cos_sin(np.arange(T), O.rope_inv_freq(spec.theta))
    for h in range(spec.num_q_heads):
        keys = O.apply_rope(qz["xk_hat"][h].astype(np.float64) @ data.k_u[h].astype(np.float64).T, cos, sin)
        ref = np.einsum("bld,bd->bl", keys, data.q[:, h].astype(np.float64))
        got = lg[:, h].cpu().numpy()
        assert O.rel_l2(got, ref) < 2e-3


def test_v_latent_matches_oracle(cuda):
    """bx's contract: P @ dequant(X_v) per head, zero outside the head's V block."""
    spec = make_spec("c1", seed=14, num_q_heads=8, batch=2, context=700)
    data = make_layer(spec)
    st = build_step(data, cuda)
    st.layer.append(st.k_new, st.v_new)
    T = spec.tokens
    rng = np.random.default_rng(0)
    p = rng.random((spec.batch, spec.num_q_heads, T)).astype(np.float32)
    p /= p.sum(-1, keepdims=True)
    got = ops.v_latent(st.layer.layout, st.layer.cache, torch.from_numpy(p).to(cuda), T).cpu().numpy()
    xv = O.quantize_layer(data.xk, data.xv, spec.context)["xv_hat"]
    vb = spec.v_block_of_kv()
    vcol = np.concatenate([[0], np.cumsum(spec.v_ranks)])
    for h in range(spec.num_q_heads):
        j = vb[h]
        ref = np.zeros((spec.batch, spec.v_rank_total))
        ref[:, vcol[j]:vcol[j + 1]] = np.einsum("bl,blr->br", p[:, h], xv[:, :, vcol[j]:vcol[j + 1]])
        assert O.rel_l2(got[:, h], ref) < 1e-3       # fp16 tensor-core operands (x_hat, p)


@pytest.mark.parametrize("cfg,over,seqs", [
    ("c1", {}, (0, 15)),                       # B=16, 32K context, 32 MHA heads, fp16
    ("c2", {}, (0, 3)),                        # GQA 32/8, B=4, 131072 context, bf16, theta 5e5
    ("c2", dict(theta=1e4, batch=2), (1,)),    # 131072 context at theta 1e4: the longest RoPE recurrence
])
def test_full_size_against_oracle(cuda, cfg, over, seqs):
    """BASELINE configurations at full size: the listed sequences against the
    oracle (fp32 output), every sequence finite, the device error word clear.
    At 131072 positions the K kernel's per-tile RoPE advance runs 512 times per
    drain thread; the oracle uses the reference's fp32 angles."""
    spec = make_spec(cfg, **over)
    st, k_u_heads, v_u = device_layer(spec, cuda, seed=1)
    L = st.layer
    L.append(st.k_new, st.v_new)
    out = torch.empty(spec.batch, spec.num_q_heads, 128, dtype=torch.float32, device=cuda)
    ops.decode_attention(L.layout, L.cache, st.q, L.k_u, L.v_u, L.inv_freq, L.scaling, L.length, out=out)
    torch.cuda.synchronize()
    assert ops.read_device_error(device=cuda) == 0
    assert torch.isfinite(out).all()
    kcol = np.concatenate([[0], np.cumsum(spec.k_ranks)[:-1]])
    # the inverse frequencies as torch computes them (HF LlamaRotaryEmbedding, which
    # the reference uses); numpy's fp32 power can differ in the last bit, which at
    # 131072 positions moves the fastest angles by ~1e-2 rad
    inv_freq = L.inv_freq.cpu().numpy()
    for b in seqs:
        xk = [st.k_lat[b:b + 1, :, c0:c0 + r].float().cpu().numpy() for c0, r in zip(kcol, spec.k_ranks)]
        xv = st.v_lat[b:b + 1].float().cpu().numpy()
        qz = O.quantize_layer(xk, xv, spec.context)
        ref = O.decode_attention(st.q[b:b + 1].float().cpu().numpy(), qz["xk_hat"],
                                 [u.float().cpu().numpy() for u in k_u_heads], qz["xv_hat"],
                                 v_u.float().cpu().numpy(), spec.k_ranks, spec.v_ranks, spec.v_block_of_kv(),
                                 inv_freq, 128 ** -0.5, dtype=np.float64)
        got = out[b:b + 1].cpu().numpy()
        err, mx = O.rel_l2(got, ref), float(np.abs(got - ref).max())
        print(f"{cfg} {over} seq {b}: rel_l2={err:.2e} max_abs={mx:.2e}")
        assert err <= REL_L2
        assert mx <= MAX_ABS
