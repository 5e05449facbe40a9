"""The CPU oracle against the golden vectors produced by the reference's own
eager module (tests/golden/make_golden.py), and the quantiser specification."""

import json
import os

import numpy as np
import pytest

import starkv_oracle as O
from starkv.synthetic import make_layer, make_spec

from conftest import GOLDEN

MANIFEST = json.load(open(os.path.join(GOLDEN, "manifest.json")))


@pytest.mark.parametrize("name", sorted(MANIFEST))
def test_oracle_matches_reference_golden(name):
    m = MANIFEST[name]
    spec = make_spec(m["config"], seed=0, **m["overrides"])
    assert spec.describe()["k_ranks"] == m["spec"]["k_ranks"]          # seeded draws are stable
    data = make_layer(spec, with_mask=m["with_mask"])
    gold = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    out = O.layer_reference(data).reshape(spec.batch, -1)
    assert O.rel_l2(out, gold["attn"]) < 5e-5
    assert np.abs(out - gold["attn"]).max() < 1e-4


def test_k_quantiser_spec():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2, 3, 50, 32)).astype(np.float32)
    x[..., 5] = 0.0                                                      # an all-zero channel
    s = O.quantize_k_scales(x)
    assert s.dtype == np.float16 and s.shape == (2, 3, 32)
    assert np.all(s[..., 5] == 1.0)
    amax = np.abs(x).max(axis=-2)
    np.testing.assert_array_equal(s[..., :5], (amax[..., :5] / np.float32(127)).astype(np.float16))
    q = O.quantize_k_codes(x, s)
    assert q.dtype == np.int8 and q.min() >= -127 and q.max() <= 127
    err = np.abs(O.dequant_k(q, s) - x)
    assert np.all(err <= s.astype(np.float32)[..., None, :] * 0.5 + 1e-6)
    # appended tokens beyond the prefill range saturate instead of wrapping
    big = x[..., :1, :] * 1000
    qb = O.quantize_k_codes(big, s)
    assert qb.max() <= 127 and qb.min() >= -127


def test_v_quantiser_spec_and_nibble_order():
    rng = np.random.default_rng(2)
    x = rng.standard_normal((4, 7, 96)).astype(np.float32)
    x[0, 0, :32] = 3.0                                                  # constant group -> scale 1
    c, s, z = O.quantize_v(x)
    assert c.shape == (4, 7, 48) and s.shape == (4, 7, 3) and z.shape == (4, 7, 3)
    assert s[0, 0, 0] == 1.0 and z[0, 0, 0] == np.float16(3.0)
    q = O.unpack_v_codes(c)
    assert q.max() <= 15
    # even channel in the low nibble (bx_quant.py:75-85)
    np.testing.assert_array_equal(c & 0x0F, q[..., 0::2])
    np.testing.assert_array_equal(c >> 4, q[..., 1::2])
    xh = O.dequant_v(c, s, z)
    step = np.repeat(s.astype(np.float32), 32, axis=-1)
    assert np.all(np.abs(xh - x) <= 0.5 * step + 2e-3 * np.abs(x) + 1e-3)


def test_rope_tables_match_hf():
    import torch
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding

    from starkv.layer import rope_inv_freq
    for theta in (1e4, 5e5):
        cfg = LlamaConfig(hidden_size=4096, num_attention_heads=32, rope_theta=theta)
        rope = LlamaRotaryEmbedding(config=cfg)
        np.testing.assert_array_equal(rope.inv_freq.numpy(), rope_inv_freq(theta).numpy())
        pos = torch.arange(0, 40000, 997)[None]
        cos, sin = rope(torch.zeros(1, dtype=torch.float32), pos)
        oc, os_ = O.rope_cos_sin(pos[0].numpy(), rope.inv_freq.numpy())
        assert np.abs(cos[0].numpy() - oc).max() < 2e-6
        assert np.abs(sin[0].numpy() - os_).max() < 2e-6


def test_bytes_accounting_c1():
    spec = make_spec("c1")
    per_tok = spec.k_rank_total + spec.v_rank_total // 2 + spec.v_rank_total // 32 * 4
    assert spec.compressed_bytes_per_token() == per_tok
    assert spec.compressed_bytes_per_step() == 16 * 32769 * per_tok + 16 * spec.k_rank_total * 2
