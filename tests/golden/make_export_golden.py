"""Golden vectors for the ragged export: the reference's own
``model.DecomposeLinear_headwise`` and ``model.export_kproj_for_triton``
(model.py:76-175, 284-325) run on a small seeded K projection (2 KV heads of
128, 48 input features), with thresholds giving (a) equal kept ranks and (b)
ragged kept ranks (where the reference truncates every head to the smallest).
Run in a container that has the reference checked out:

    python tests/golden/make_export_golden.py /path/to/reference
"""

import os
import sys

import numpy as np
import torch
import torch.nn as nn

ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("STARKV_REFERENCE", "")
sys.path.insert(0, ref)
import model  # noqa: E402  (the reference's module)

torch.manual_seed(11)
lin = nn.Linear(48, 256, bias=False)
lin._num_heads = 2
lin._head_dim = 128
dec = model.DecomposeLinear_headwise(lin)
out = {"U": dec.U.weight.detach().numpy(), "V": dec.V.weight.detach().numpy()}
for case, keep in (("equal", (32, 32)), ("ragged", (32, 16))):
    for h, sb in enumerate(dec.Sigma_blocks):
        d = sb.diag.detach()
        alpha = float((d.sort(descending=True).values[keep[h] - 1] + d.sort(descending=True).values[keep[h]]) / 2)
        sb.soft_thres_layer.alpha.data.fill_(alpha)
        out[f"{case}_diag{h}"] = d.numpy()
        out[f"{case}_alpha{h}"] = np.float32(alpha)
    vs, u = model.export_kproj_for_triton(dec, dtype=torch.float32)
    out[f"{case}_VS"] = vs.weight.detach().numpy()
    out[f"{case}_Uref"] = u.numpy()
np.savez_compressed(os.path.join(os.path.dirname(os.path.abspath(__file__)), "export_k.npz"), **out)
print("wrote export_k.npz")
