"""Seeded synthetic layers for the STAR-KV decode step.

The reference measures on real checkpoints (longchat / Llama-2-7B exports) that
are not available here; these generators stand in with the shapes, rank
distributions and value distributions of the benchmark configurations:

* K latents X_k[h] ~ N(0, 1) per KV head (T x r_h), V latents ~ N(0, 1)
  (T x sum r_b); for quantised configurations 1% of the latent channels are
  scaled by 8 (outlier channels) before quantisation;
* K up-projection U_k[h] (128 x r_h) ~ N(0, 1/r_h); V up-projection block
  (128 x r_b per KV head of the block) ~ N(0, 1/r_b), zero outside the block;
* rotated query ~ N(0, 1).

Ranks are drawn per KV head / per V block from the configuration's rank set
with ``numpy.random.default_rng(seed)``, so every machine draws the same ranks.
"""

from __future__ import annotations

import dataclasses
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np

DTYPES = ("float32", "float16", "bfloat16")


@dataclass
class LayerSpec:
    """Shape of one compressed-KV attention layer at one decode step."""

    batch: int
    context: int                 # cached tokens before the step (positions 0..context-1)
    num_q_heads: int
    num_kv_heads: int
    theta: float
    k_ranks: List[int]           # per KV head, multiples of 16
    v_ranks: List[int]           # per V block, multiples of 32
    v_block_kv: List[int]        # KV heads per V block (contiguous head ranges)
    dtype: str = "float16"
    quantized: bool = True
    head_dim: int = 128
    name: str = "custom"
    seed: int = 0

    @property
    def tokens(self) -> int:
        """Tokens attended by the step: the cache plus the appended token."""
        return self.context + 1

    @property
    def num_v_blocks(self) -> int:
        return len(self.v_ranks)

    @property
    def k_rank_total(self) -> int:
        return int(sum(self.k_ranks))

    @property
    def v_rank_total(self) -> int:
        return int(sum(self.v_ranks))

    def v_block_of_kv(self) -> List[int]:
        out = []
        for j, n in enumerate(self.v_block_kv):
            out += [j] * n
        return out

    def compressed_bytes_per_token(self) -> int:
        """Compressed-cache bytes one decode step reads per (sequence, token).

        Quantised: int8 K codes (1 B per channel) + int4 V codes (0.5 B per
        channel) + fp16 scale and zero point per 32 V channels.  Unquantised:
        latents in their storage dtype."""
        if self.quantized:
            return self.k_rank_total + self.v_rank_total // 2 + (self.v_rank_total // 32) * 4
        es = 4 if self.dtype == "float32" else 2
        return (self.k_rank_total + self.v_rank_total) * es

    def compressed_bytes_per_step(self) -> int:
        b = self.batch * self.tokens * self.compressed_bytes_per_token()
        if self.quantized:
            b += self.batch * self.k_rank_total * 2        # per-channel K scales
        return b

    def flops_per_step(self) -> int:
        """Algorithmic FLOPs: K reconstruction (2*128*r per KV-head token), q.k per
        query head, and P.X_v per query head."""
        grp = self.num_q_heads // self.num_kv_heads
        vb = self.v_block_of_kv()
        f = 0
        for kv in range(self.num_kv_heads):
            f += 2 * self.head_dim * self.k_ranks[kv]
            f += grp * (2 * self.head_dim + 2 * self.v_ranks[vb[kv]])
        return self.batch * self.tokens * f

    def describe(self) -> dict:
        d = dataclasses.asdict(self)
        d["tokens"] = self.tokens
        return d


def _draw(rng, choices, n):
    return [int(x) for x in rng.choice(np.asarray(choices), size=n)]


def make_spec(name: str, seed: int = 0, **over) -> LayerSpec:
    """Benchmark configurations (1, 2, 4) with seeded ranks."""
    rng = np.random.default_rng(seed)
    if name in ("c0", "c1", "c4"):
        hq = hkv = over.pop("num_q_heads", 32)
        hkv = over.pop("num_kv_heads", hq)
        kset = [16, 32, 48] if name == "c4" else [16, 32, 48, 64, 80, 96]
        nblk = hkv // 4
        spec = LayerSpec(
            batch=1 if name == "c0" else 16,
            context=2048 if name == "c0" else 32768,
            num_q_heads=hq, num_kv_heads=hkv, theta=1e4,
            k_ranks=_draw(rng, kset, hkv),
            v_ranks=_draw(rng, [64, 128, 192], nblk),
            v_block_kv=[4] * nblk,
            dtype="float32" if name == "c0" else "float16",
            quantized=(name != "c0"), name=name, seed=seed)
    elif name == "c2":
        hq = over.pop("num_q_heads", 32)
        hkv = over.pop("num_kv_heads", 8)
        nblk = hkv // 2
        spec = LayerSpec(
            batch=4, context=131072, num_q_heads=hq, num_kv_heads=hkv, theta=5e5,
            k_ranks=_draw(rng, [32, 48, 64, 80, 96], hkv),
            v_ranks=_draw(rng, [64, 128, 192], nblk),
            v_block_kv=[2] * nblk, dtype="bfloat16", quantized=True, name=name, seed=seed)
    else:
        raise ValueError(f"unknown configuration {name!r}")
    for k, v in over.items():
        setattr(spec, k, v)
    return spec


@dataclass
class LayerData:
    """Float32 values of one synthetic layer (numpy, already rounded to ``spec.dtype``)."""

    spec: LayerSpec
    xk: List[np.ndarray]          # per KV head (B, T, r_h); token T-1 is the appended one
    xv: np.ndarray                # (B, T, sum r_b)
    k_u: List[np.ndarray]         # per KV head (128, r_h)
    v_u: np.ndarray               # (Hkv*128, sum r_b), block diagonal
    q: np.ndarray                 # (B, Hq, 128) rotated query
    mask: Optional[np.ndarray] = None   # (B, T) additive, or None


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` (via torch for bfloat16) and back to float32."""
    if dtype == "float32":
        return x.astype(np.float32)
    if dtype == "float16":
        return x.astype(np.float16).astype(np.float32)
    import torch
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(torch.bfloat16).float().numpy()


def make_layer(spec: LayerSpec, seed: Optional[int] = None, with_mask: bool = False) -> LayerData:
    rng = np.random.default_rng(spec.seed + 1000 if seed is None else seed)
    B, T = spec.batch, spec.tokens
    D = spec.head_dim
    outl = spec.quantized

    def lat(shape):
        x = rng.standard_normal(shape, dtype=np.float32)
        if outl:
            r = shape[-1]
            n = max(1, int(round(0.01 * r)))
            ch = rng.choice(r, size=n, replace=False)
            x[..., ch] *= 8.0
        return round_to(x, spec.dtype)

    xk = [lat((B, T, r)) for r in spec.k_ranks]
    xv = lat((B, T, spec.v_rank_total))
    k_u = [round_to(rng.standard_normal((D, r), dtype=np.float32) / np.sqrt(r), spec.dtype)
           for r in spec.k_ranks]
    v_u = np.zeros((spec.num_kv_heads * D, spec.v_rank_total), dtype=np.float32)
    vb = spec.v_block_of_kv()
    vcol = np.concatenate([[0], np.cumsum(spec.v_ranks)])
    for kv in range(spec.num_kv_heads):
        j = vb[kv]
        r = spec.v_ranks[j]
        v_u[kv * D:(kv + 1) * D, vcol[j]:vcol[j + 1]] = round_to(
            rng.standard_normal((D, r), dtype=np.float32) / np.sqrt(r), spec.dtype)
    q = round_to(rng.standard_normal((B, spec.num_q_heads, D), dtype=np.float32), spec.dtype)
    mask = None
    if with_mask:
        mask = np.zeros((B, T), dtype=np.float32)
        for b in range(B):
            npad = int(rng.integers(0, max(1, T // 5)))
            mask[b, :npad] = -1e9                      # left padding
            mask[b, npad:] = rng.uniform(-2.0, 0.0, size=T - npad).astype(np.float32) * (b % 2)
    return LayerData(spec, xk, xv, k_u, v_u, q, mask)
