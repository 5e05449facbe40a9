"""Generate the golden decode-attention vectors from the reference's own eager code.

Run here (where the reference tree is mounted) with::

    python tests/golden/make_golden.py [--ref /path/to/STAR-KV]

It imports the reference's ``LlamaLoRaAttention_headwise.LlamaCustomAttention``
(eager branch: ``triton_kernel = False``, ``reorder = True``) and, for GQA, its
``model._patched_attn_forward`` decode branch, and runs one decode step on CPU in
fp32 for each case below.  Inputs are regenerated from seeds by
``starkv.synthetic`` (numpy PCG64, identical on every machine), so a fixture only
stores the case parameters and the reference's outputs:

* ``attn``  — the per-head attention output fed to ``o_proj`` (B, Hq*128),
  captured with a forward pre-hook on ``o_proj``;
* ``out``   — the module's output after ``o_proj`` (B, hidden).

Ragged per-head K ranks are zero-padded to the largest rank and block-wise V is
a block-diagonal ``v_proj.U`` — the reference layout for the same math.  For
quantised cases the reference runs on the dequantised cache (the quantiser
module the reference imports is absent from its tree); the cache object passed
as ``past_key_values`` quantises the appended token with the prefill's K scales
before concatenating, as the B200 cache does.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(REPO, "star-kv_b200"), os.path.join(REPO, "oracle")]

sys.path.insert(0, os.path.dirname(HERE))
from starkv.synthetic import make_spec, make_layer  # noqa: E402
import starkv_oracle as O  # noqa: E402
from golden_inputs import build_module_inputs, prefill_cache  # noqa: E402

# name -> (config, overrides, with_mask, gqa)
CASES = {
    "c0_full": ("c0", dict(), False),
    "c0_small": ("c0", dict(num_q_heads=8, batch=2, context=300), False),
    "c0_small_mask": ("c0", dict(num_q_heads=8, batch=2, context=257), True),
    "c1_small": ("c1", dict(num_q_heads=8, batch=2, context=515), False),
    "c1_tiny": ("c1", dict(num_q_heads=4, batch=3, context=1), False),
    "c2_small": ("c2", dict(num_q_heads=16, num_kv_heads=4, batch=2, context=640), False),
}


class _StepCache:
    """Minimal ``Cache`` stand-in exposing the ``update(k, v, layer_idx)`` contract
    the reference calls (headwise.py:99, model.py:419)."""

    def __init__(self, k_prev, v_prev, k_scales=None):
        self.k_prev, self.v_prev, self.k_scales = k_prev, v_prev, k_scales

    def update(self, k_new, v_new, layer_idx):
        import torch
        if self.k_scales is not None:
            kn = k_new.detach().numpy()                                   # (B, H, 1, rmax)
            kq = O.quantize_k_codes(kn, self.k_scales)
            kn = O.dequant_k(kq, self.k_scales)
            vn = v_new.detach().numpy()                                   # (B, 1, R)
            c, s, z = O.quantize_v(vn)
            vn = O.dequant_v(c, s, z)
            k_new = torch.from_numpy(kn.astype(np.float32))
            v_new = torch.from_numpy(vn.astype(np.float32))
        return torch.cat([self.k_prev, k_new], dim=-2), torch.cat([self.v_prev, v_new], dim=-2)


def run_case(name, ref_dir):
    import torch
    import torch.nn as nn
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding

    cfg_name, over, with_mask = CASES[name]
    spec = make_spec(cfg_name, seed=0, **over)
    data = make_layer(spec, with_mask=with_mask)
    rng = np.random.default_rng(4242)
    D = spec.head_dim
    hidden = spec.num_q_heads * D
    rmax = max(spec.k_ranks)
    h, wq, vs_k, vs_v, k_u, wo = build_module_inputs(spec, data, rng)

    sys.path.insert(0, ref_dir)
    import LlamaLoRaAttention_headwise as ref_attn
    ref_attn.triton_kernel = False
    ref_attn.reorder = True

    config = LlamaConfig(hidden_size=hidden, num_attention_heads=spec.num_q_heads,
                         num_key_value_heads=spec.num_kv_heads, intermediate_size=4 * hidden,
                         rope_theta=spec.theta, max_position_embeddings=max(4096, spec.tokens + 1),
                         attention_bias=False, head_dim=D)
    mod = ref_attn.LlamaCustomAttention(config, layer_idx=0, decomp_goup_num=spec.num_q_heads).float().eval()
    with torch.no_grad():
        mod.q_proj.weight.copy_(torch.from_numpy(wq))
        mod.o_proj.weight.copy_(torch.from_numpy(wo))
    kvs = nn.Linear(hidden, spec.num_kv_heads * rmax, bias=False)
    kvs.weight = nn.Parameter(torch.from_numpy(vs_k))
    kp = nn.Module()
    kp.VS = kvs
    kp.register_buffer("U", torch.from_numpy(k_u))
    vvs = nn.Linear(hidden, spec.v_rank_total, bias=False)
    vvs.weight = nn.Parameter(torch.from_numpy(vs_v))
    vu = nn.Linear(spec.v_rank_total, spec.num_kv_heads * D, bias=False)
    vu.weight = nn.Parameter(torch.from_numpy(data.v_u))
    vp = nn.Module()
    vp.VS = vvs
    vp.U = vu
    mod.k_proj = kp
    mod.v_proj = vp

    L = spec.context
    B = spec.batch
    kprev, xv_prev, ks = prefill_cache(spec, data)
    cache = _StepCache(torch.from_numpy(kprev), torch.from_numpy(xv_prev), ks)

    rope = LlamaRotaryEmbedding(config=config)
    pos = torch.arange(spec.tokens).unsqueeze(0).expand(B, -1)
    x = torch.from_numpy(h)
    cos, sin = rope(x, pos)                                                 # positions 0..L
    mask = None
    if data.mask is not None:
        mask = torch.from_numpy(data.mask)[:, None, None, :]
    captured = {}
    hook = mod.o_proj.register_forward_pre_hook(lambda m, a: captured.__setitem__("attn", a[0].detach().clone()))
    with torch.no_grad():
        if spec.num_q_heads == spec.num_kv_heads:
            out, _ = mod(x, (cos, sin), mask, pos[:, -1:], past_key_values=cache)
        else:
            import model as ref_model                                        # GQA: model.py:450-487
            ref_attn.triton_kernel = False
            out, _ = ref_model._patched_attn_forward(mod, x, (cos, sin), mask, pos[:, -1:],
                                                     past_key_values=cache)
    hook.remove()
    sys.path.remove(ref_dir)
    return spec, dict(attn=captured["attn"].reshape(B, -1).numpy().astype(np.float32),
                      out=out.reshape(B, -1).numpy().astype(np.float32),
                      wo_seed=np.int64(4242))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("STARKV_REFERENCE"),
                    help="checkout of the reference (or set STARKV_REFERENCE)")
    ap.add_argument("--only", nargs="*")
    args = ap.parse_args()
    manifest = {}
    for name in (args.only or CASES):
        if not args.ref:
            ap.error("pass --ref or set STARKV_REFERENCE to the reference checkout")
        spec, res = run_case(name, args.ref)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **res)
        manifest[name] = dict(config=CASES[name][0], overrides=CASES[name][1], with_mask=CASES[name][2],
                              spec=spec.describe())
        print(name, res["attn"].shape, os.path.getsize(path))
    mpath = os.path.join(HERE, "manifest.json")
    old = json.load(open(mpath)) if os.path.exists(mpath) else {}
    old.update(manifest)
    with open(mpath, "w") as f:
        json.dump(old, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
