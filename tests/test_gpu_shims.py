"""The reference-interface drop-in modules on the GPU against the oracle:
``quant_utils`` (split int8 / int4 quantiser, bit-exact), ``bx_quant.bx`` and
``abx_rope_batched_quant.abx`` (within the north-star tolerance)."""

import os
import sys

import numpy as np
import pytest
import torch

import starkv_oracle as O
from conftest import ROOT

sys.path.insert(0, os.path.join(ROOT, "star-kv_b200"))
import abx_rope_batched_quant  # noqa: E402
import bx_quant  # noqa: E402
import quant_utils  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape,split", [((2, 3, 77, 96), 16), ((4, 333, 832), 256), ((5, 40), 0), ((5, 40), 40),
                                         ((3, 9, 37), 16)])
def test_split_quantiser_bit_exact(cuda, shape, split):
    rng = np.random.default_rng(1)
    x = rng.standard_normal(shape).astype(np.float32) * rng.uniform(0.1, 5.0, size=shape[:-1] + (1,))
    x[..., 3] *= 8.0
    if len(shape) > 2:
        x[0, 0] = 0.0                                  # a zero row: scale 1
    xt = torch.from_numpy(x).to(cuda, torch.float16)
    xh = xt.float().cpu().numpy()
    got = quant_utils.quantize_r_split_int8_int4_packed(xt, split)
    want = O.quantize_split(xh, split)
    assert got[4] == want[4]
    for g, w in zip(got[:4], want[:4]):
        np.testing.assert_array_equal(g.cpu().numpy(), w)
    np.testing.assert_array_equal(quant_utils.unpack_uint8_to_int4_signed(got[2], got[4]).cpu().numpy(),
                                  O.unpack_int4_signed(want[2], want[4]))


def test_bx_shim_matches_oracle(cuda):
    rng = np.random.default_rng(2)
    B, H, L, up, R = 2, 32, 700, 256, 832
    x = rng.standard_normal((B, L, R)).astype(np.float32)
    xt = torch.from_numpy(x).to(cuda, torch.float16)
    # the reference kernel reads both blocks as nibbles with per-token scales
    _, _, lo_up, s_up, _ = quant_utils.quantize_r_split_int8_int4_packed(xt[..., :up], 0)
    _, _, lo_lo, s_lo, _ = quant_utils.quantize_r_split_int8_int4_packed(xt[..., up:], 0)
    p = rng.random((B, H, L)).astype(np.float32)
    p /= p.sum(-1, keepdims=True)
    pt = torch.from_numpy(p).to(cuda, torch.float16)
    got = bx_quant.bx(pt, lo_up, lo_lo, s_up, s_lo, original_rank=R, upper_rank=up).float().cpu().numpy()
    deq = np.concatenate([O.unpack_int4_signed(lo_up.cpu().numpy(), up) * s_up.float().cpu().numpy(),
                          O.unpack_int4_signed(lo_lo.cpu().numpy(), R - up) * s_lo.float().cpu().numpy()], axis=-1)
    ref = np.einsum("bhl,blr->bhr", pt.float().cpu().numpy(), deq)
    assert O.rel_l2(got, ref) <= 2e-3


def test_abx_quant_shim_matches_oracle(cuda):
    rng = np.random.default_rng(3)
    B, Hq, Hkv, L, r = 2, 8, 4, 500, 64
    lat = rng.standard_normal((B, Hkv, L, r)).astype(np.float32)
    up_q, s_up, lo_q, s_lo, r4 = quant_utils.quantize_r_split_int8_int4_packed(
        torch.from_numpy(lat).to(cuda, torch.float16), 16)
    u = (rng.standard_normal((Hkv, 128, r)) / np.sqrt(r)).astype(np.float16)
    q = rng.standard_normal((B, Hq, 1, 128)).astype(np.float16)
    rep = Hq // Hkv
    got = abx_rope_batched_quant.abx(torch.from_numpy(q).to(cuda), torch.from_numpy(u).to(cuda).transpose(-1, -2),
                                     up_q.repeat_interleave(rep, dim=1), lo_q.repeat_interleave(rep, dim=1),
                                     s_up, s_lo, r4).float().cpu().numpy()
    deq = np.concatenate([up_q.cpu().numpy() * s_up.float().cpu().numpy(),
                          O.unpack_int4_signed(lo_q.cpu().numpy(), r4) * s_lo.float().cpu().numpy()], axis=-1)
    deq = deq.astype(np.float16).astype(np.float64)
    cos, sin = O.rope_cos_sin(np.arange(L), O.rope_inv_freq(1e4))
    for h in range(Hq):
        keys = O.apply_rope(deq[:, h // rep] @ u[h // rep].astype(np.float64).T, cos, sin)
        ref = np.einsum("bld,bd->bl", keys, q[:, h, 0].astype(np.float64))
        assert O.rel_l2(got[:, h, 0], ref) <= 2e-3
