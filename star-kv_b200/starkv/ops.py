"""Torch-facing wrappers of the libstarkv C ABI.

Every op launches on the current torch CUDA stream, takes and returns torch
tensors, and goes through ``libstarkv.so``; there is no CPU path.  Device
memory (caches, workspaces, outputs) comes from torch's allocator here in the
host layer — the C ABI itself never allocates.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import List, Optional, Sequence

import torch

from . import _lib
from ._lib import BF16, F16, F32, DecodeArgs, Layout, check, load

_DT = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}
_TORCH = {F32: torch.float32, F16: torch.float16, BF16: torch.bfloat16}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DT[dt]
    except KeyError:
        raise _lib.StarKVError(f"unsupported dtype {dt}") from None


def _ptr(t: Optional[torch.Tensor]):
    if t is None:
        return None
    if not t.is_cuda:
        raise _lib.StarKVError("libstarkv ops take CUDA tensors")
    return C.c_void_p(t.data_ptr())


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _require(t: torch.Tensor, name: str, dtype=None, numel=None, align=16):
    if not t.is_cuda:
        raise _lib.StarKVError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise _lib.StarKVError(f"{name} must be contiguous")
    if dtype is not None and t.dtype != dtype:
        raise _lib.StarKVError(f"{name} must be {dtype}, got {t.dtype}")
    if numel is not None and t.numel() != numel:
        raise _lib.StarKVError(f"{name} must have {numel} elements, got {t.numel()}")
    if t.data_ptr() % align:
        raise _lib.StarKVError(f"{name} must be {align}-byte aligned")


def make_layout(batch: int, num_q_heads: int, num_kv_heads: int, k_ranks: Sequence[int],
                v_ranks: Sequence[int], v_block_kv: Sequence[int], capacity: int, quantized: bool,
                latent_dtype: torch.dtype, k_offsets: Optional[Sequence[int]] = None,
                k_batch_strides: Optional[Sequence[int]] = None, k_tiled: Optional[bool] = None) -> Layout:
    """Build a ``starkv_layout``.  Default K layout: head h is a contiguous
    (B, capacity, r_h) region at offset B*capacity*sum(r_<h), tiled (128-slot
    tiles of 16-byte column chunks) with the capacity rounded up to a multiple
    of 128.  Explicit offsets / strides (the reference's (B, Hkv, L, r) tensor)
    default to the row-major layout."""
    if k_tiled is None:
        k_tiled = k_offsets is None and k_batch_strides is None
    if k_tiled:
        capacity = (capacity + 127) // 128 * 128
    L = Layout()
    L.abi_version = _lib.ABI_VERSION
    L.batch, L.num_q_heads, L.num_kv_heads, L.head_dim = batch, num_q_heads, num_kv_heads, 128
    L.num_v_blocks = len(v_ranks)
    L.capacity = capacity
    L.quantized = int(bool(quantized))
    L.latent_dtype = dtype_code(latent_dtype)
    L.k_tiled = int(bool(k_tiled))
    col = 0
    for h, r in enumerate(k_ranks):
        L.k_rank[h] = r
        L.k_col[h] = col
        L.k_offset[h] = batch * capacity * col if k_offsets is None else k_offsets[h]
        L.k_batch_stride[h] = capacity * r if k_batch_strides is None else k_batch_strides[h]
        col += r
    L.k_rank_total = col
    vcol, kv = 0, 0
    for j, (r, n) in enumerate(zip(v_ranks, v_block_kv)):
        L.v_rank[j], L.v_col[j], L.v_first_kv[j], L.v_num_kv[j] = r, vcol, kv, n
        vcol += r
        kv += n
    L.v_rank_total = vcol
    check(load().starkv_validate_layout(C.byref(L)), "layout validation")
    return L


def layout_from_spec(spec, capacity: Optional[int] = None) -> Layout:
    """Layout of a ``starkv.synthetic.LayerSpec``."""
    return make_layout(spec.batch, spec.num_q_heads, spec.num_kv_heads, spec.k_ranks, spec.v_ranks,
                       spec.v_block_kv, capacity or spec.tokens, spec.quantized, _TORCH[dtype_code(
                           getattr(torch, spec.dtype))])


class LatentCache:
    """Preallocated latent cache of one layer (the static replacement of the
    reference's DynamicCache entries, LlamaLoRaAttention_headwise.py:98-102 /
    LlamaLoRaAttention_headwise_quant.py:119-132).

    Quantised: ``k_cache`` int8 codes, ``k_scales`` fp16 (B, sum r_h),
    ``v_cache`` uint8 packed int4 (B, capacity, R/2), ``v_params`` fp16
    (B, capacity, R/32, 2) = (scale, zero).  Unquantised: latents in the layout's
    dtype.  ``length`` is the number of filled slots."""

    def __init__(self, layout: Layout, device=None):
        self.layout = layout
        dev = torch.device(device or "cuda")
        B, cap = layout.batch, layout.capacity
        K, R = layout.k_rank_total, layout.v_rank_total
        if layout.quantized:
            self.k_cache = torch.zeros(B * cap * K, dtype=torch.int8, device=dev)
            self.k_scales = torch.ones(B * K, dtype=torch.float16, device=dev)
            self.v_cache = torch.zeros(B, cap, R // 2, dtype=torch.uint8, device=dev)
            self.v_params = torch.zeros(B, cap, R // 32, 2, dtype=torch.float16, device=dev)
        else:
            dt = _TORCH[layout.latent_dtype]
            self.k_cache = torch.zeros(B * cap * K, dtype=dt, device=dev)
            self.k_scales = None
            self.v_cache = torch.zeros(B, cap, R, dtype=dt, device=dev)
            self.v_params = None
        self.length = 0

    @property
    def latent_dtype(self) -> torch.dtype:
        return _TORCH[self.layout.latent_dtype]

    def prefill(self, k_lat: torch.Tensor, v_lat: torch.Tensor):
        """k_lat (B, T, sum r_h), v_lat (B, T, R) in the latent dtype; fills slots [0, T)
        and (quantised) fixes the per-channel K scales."""
        L = self.layout
        T = k_lat.shape[1]
        _require(k_lat, "k_lat", self.latent_dtype, L.batch * T * L.k_rank_total)
        _require(v_lat, "v_lat", self.latent_dtype, L.batch * T * L.v_rank_total)
        check(load().starkv_quantize_prefill(C.byref(L), _ptr(k_lat), _ptr(v_lat), T, _ptr(self.k_cache),
                                             _ptr(self.k_scales), _ptr(self.v_cache), _ptr(self.v_params),
                                             _stream()), "starkv_quantize_prefill")
        self.length = T

    def append(self, k_lat: torch.Tensor, v_lat: torch.Tensor):
        """Quantise (with the existing K scales) and write T new tokens at slot ``length``."""
        L = self.layout
        T = k_lat.shape[1]
        _require(k_lat, "k_lat", self.latent_dtype, L.batch * T * L.k_rank_total, align=2)
        _require(v_lat, "v_lat", self.latent_dtype, L.batch * T * L.v_rank_total, align=2)
        check(load().starkv_append(C.byref(L), _ptr(k_lat), _ptr(v_lat), T, self.length, _ptr(self.k_cache),
                                   _ptr(self.k_scales), _ptr(self.v_cache), _ptr(self.v_params), _stream()),
              "starkv_append")
        self.length += T

    def project_append(self, hidden: torch.Tensor, vs_k: torch.Tensor, vs_v: torch.Tensor,
                       return_latents: bool = False):
        """One decode token per sequence straight from the hidden state: the fused
        ``k_proj.VS`` / ``v_proj.VS`` projection + quantise-append at slot ``length``
        (``starkv_project_append``).  hidden (B, 1, hidden) or (B, hidden); vs_k
        (sum r_h, hidden); vs_v (R, hidden); all in the latent dtype.  With
        ``return_latents`` the rounded latents (B, 1, sum r_h) / (B, 1, R) are returned."""
        L = self.layout
        H = hidden.shape[-1]
        dt = self.latent_dtype
        _require(hidden, "hidden", dt, L.batch * H)
        _require(vs_k, "vs_k", dt, L.k_rank_total * H)
        _require(vs_v, "vs_v", dt, L.v_rank_total * H)
        k_out = v_out = None
        if return_latents:
            k_out = torch.empty(L.batch, 1, L.k_rank_total, dtype=dt, device=hidden.device)
            v_out = torch.empty(L.batch, 1, L.v_rank_total, dtype=dt, device=hidden.device)
        check(load().starkv_project_append(C.byref(L), _ptr(hidden), H, _ptr(vs_k), _ptr(vs_v), self.length,
                                           _ptr(self.k_cache), _ptr(self.k_scales), _ptr(self.v_cache),
                                           _ptr(self.v_params), _ptr(k_out), _ptr(v_out), _stream()),
              "starkv_project_append")
        self.length += 1
        return (k_out, v_out) if return_latents else None

    # ---- host views for tests / export
    def k_head(self, h: int) -> torch.Tensor:
        """(B, capacity, r_h) row-major copy (tiled layout) or view (row-major) of KV head h."""
        L = self.layout
        r = L.k_rank[h]
        n = L.batch * L.capacity * r
        flat = self.k_cache[L.k_offset[h]:L.k_offset[h] + n]
        if not L.k_tiled:
            return flat.view(L.batch, L.capacity, r)
        per = 16 // flat.element_size()
        t = flat.view(L.batch, L.capacity // 128, r // per, 128, per)
        return t.permute(0, 1, 3, 2, 4).reshape(L.batch, L.capacity, r)


_WORKSPACES = {}


def workspace(nbytes: int, device) -> torch.Tensor:
    """Per-device grow-only scratch buffer (zeroed on allocation: its first word is
    the kernels' device error flag)."""
    dev = torch.device(device)
    key = (dev.type, dev.index)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=dev)
        _WORKSPACES[key] = ws
    return ws


def auto_splits(layout: Layout, num_tokens: int) -> int:
    """Sequence splits the decode step picks for this layout and token count."""
    return int(load().starkv_auto_splits(C.byref(layout), int(num_tokens)))


def workspace_size(layout: Layout, num_tokens: int, num_splits: int = 0) -> int:
    n = C.c_size_t(0)
    check(load().starkv_decode_workspace_size(C.byref(layout), num_tokens, num_splits, C.byref(n)),
          "starkv_decode_workspace_size")
    return int(n.value)


def _decode_args(layout, cache, q, k_u, v_u, inv_freq, scaling, num_tokens, mask, out, ws, num_splits):
    a = DecodeArgs()
    a.q, a.q_dtype = _ptr(q), dtype_code(q.dtype)
    a.w_dtype = dtype_code(k_u.dtype)
    a.k_u, a.v_u = _ptr(k_u), _ptr(v_u) if v_u is not None else None
    a.inv_freq = _ptr(inv_freq)
    a.mask = _ptr(mask)
    a.scaling = float(scaling)
    a.num_tokens = int(num_tokens)
    a.k_cache, a.k_scales = _ptr(cache.k_cache), _ptr(cache.k_scales)
    a.v_cache, a.v_params = _ptr(cache.v_cache), _ptr(cache.v_params)
    a.out = _ptr(out)
    a.out_dtype = dtype_code(out.dtype) if out is not None else 0
    a.num_splits = int(num_splits)
    a.workspace = _ptr(ws)
    a.workspace_bytes = ws.numel() if ws is not None else 0
    return a


def decode_attention(layout: Layout, cache: LatentCache, q: torch.Tensor, k_u: torch.Tensor,
                     v_u: torch.Tensor, inv_freq: torch.Tensor, scaling: float, num_tokens: Optional[int] = None,
                     mask: Optional[torch.Tensor] = None,
                     out: Optional[torch.Tensor] = None, num_splits: int = 0,
                     ws: Optional[torch.Tensor] = None, events=None) -> torch.Tensor:
    """One decode step of compressed-KV attention over cache slots [0, num_tokens).

    q: (B, Hq, 128) rotated query; k_u: packed K up-projections (head h = (128, r_h)
    at element 128*k_col[h]; the reference's contiguous k_proj.U); v_u:
    v_proj.U.weight (Hkv*128, R).  Returns per-head outputs (B, Hq, 128)."""
    T = cache.length if num_tokens is None else num_tokens
    B, Hq = layout.batch, layout.num_q_heads
    _require(q, "q", None, B * Hq * 128, align=4)
    _require(k_u, "k_u", None, 128 * layout.k_rank_total, align=4)
    _require(v_u, "v_u", k_u.dtype, layout.num_kv_heads * 128 * layout.v_rank_total, align=4)
    if mask is not None:
        _require(mask, "mask", torch.float32, B * T, align=4)
    if out is None:
        out = torch.empty(B, Hq, 128, dtype=q.dtype, device=q.device)
    if ws is None:
        ws = workspace(workspace_size(layout, T, num_splits), q.device)
    _require(inv_freq, "inv_freq", torch.float32, 64, align=4)
    a = _decode_args(layout, cache, q, k_u, v_u, inv_freq, scaling, T, mask, out, ws, num_splits)
    if events is not None:
        # torch creates CUDA events lazily: record each once to obtain its handle
        for e in events:
            if not e.cuda_event:
                e.record()
        # four torch.cuda.Event(enable_timing=True): before K, after K, after V, after the merge
        arr = (C.c_void_p * 4)(*[C.c_void_p(e.cuda_event) for e in events])
        a.events = C.cast(arr, C.POINTER(C.c_void_p))
    check(load().starkv_decode_attention(C.byref(layout), C.byref(a), _stream()), "starkv_decode_attention")
    return out


def decode_attention_static(layout: Layout, cache: LatentCache, q: torch.Tensor, k_u: torch.Tensor,
                            v_u: torch.Tensor, inv_freq: torch.Tensor, scaling: float, num_tokens: int,
                            out: torch.Tensor, mask: Optional[torch.Tensor] = None, num_splits: int = 0) -> torch.Tensor:
    """``decode_attention`` through ``starkv_decode_attention_static``: for callers that
    cannot allocate device memory during the step, the library's fixed static scratch
    replaces the workspace.  ``out`` must be provided (nothing is allocated here)."""
    _require(inv_freq, "inv_freq", torch.float32, 64, align=4)
    a = _decode_args(layout, cache, q, k_u, v_u, inv_freq, scaling, num_tokens, mask, out, None, num_splits)
    check(load().starkv_decode_attention_static(C.byref(layout), C.byref(a), _stream()),
          "starkv_decode_attention_static")
    return out


def static_read_device_error() -> int:
    """Read and clear the device error word of the static scratch used by
    ``decode_attention_static`` (synchronises)."""
    code = C.c_int(0)
    check(load().starkv_static_read_device_error(C.byref(code), _stream()), "starkv_static_read_device_error")
    return int(code.value)


def k_logits(layout: Layout, cache: LatentCache, q: torch.Tensor, k_u: torch.Tensor, inv_freq: torch.Tensor,
             num_tokens: int, num_splits: int = 0) -> torch.Tensor:
    """logits[b, qh, l] = q . RoPE_l(X_k @ U^T), unscaled fp32 (B, Hq, num_tokens) — abx's contract."""
    B, Hq = layout.batch, layout.num_q_heads
    logits = torch.empty(B, Hq, num_tokens, dtype=torch.float32, device=q.device)
    _require(inv_freq, "inv_freq", torch.float32, 64, align=4)
    ws = workspace(workspace_size(layout, num_tokens, num_splits), q.device)
    a = _decode_args(layout, cache, q, k_u, None, inv_freq, 1.0, num_tokens, None, None, ws, num_splits)
    check(load().starkv_k_logits(C.byref(layout), C.byref(a), _ptr(logits), _stream()), "starkv_k_logits")
    return logits


def v_latent(layout: Layout, cache: LatentCache, probs: torch.Tensor, num_tokens: int) -> torch.Tensor:
    """P @ dequant(X_v) per head, in latent space — bx's contract: (B, Hq, R) fp32."""
    B, Hq = layout.batch, layout.num_q_heads
    _require(probs, "probs", torch.float32, B * Hq * num_tokens, align=4)
    out = torch.empty(B, Hq, layout.v_rank_total, dtype=torch.float32, device=probs.device)
    check(load().starkv_v_latent(C.byref(layout), _ptr(probs), num_tokens, _ptr(cache.v_cache),
                                 _ptr(cache.v_params), _ptr(out), _stream()), "starkv_v_latent")
    return out


def quantize_split(x: torch.Tensor, split_r: int):
    """The reference's split quantiser (``starkv_quantize_split``): x (..., r) ->
    (up_q int8 (..., split_r), s_up fp16 (..., 1), lo_q uint8 (..., ceil(r4/2)),
    s_lo fp16 (..., 1), r4 = r - split_r)."""
    if not x.is_cuda:
        raise _lib.StarKVError("quantize_split takes CUDA tensors")
    x = x.contiguous()
    r = x.shape[-1]
    split_r = min(int(split_r), r)
    r4 = r - split_r
    lead = x.shape[:-1]
    rows = x.numel() // r if r else 0
    up = torch.empty(*lead, split_r, dtype=torch.int8, device=x.device)
    s_up = torch.ones(*lead, 1, dtype=torch.float16, device=x.device)
    lo = torch.empty(*lead, (r4 + 1) // 2, dtype=torch.uint8, device=x.device)
    s_lo = torch.ones(*lead, 1, dtype=torch.float16, device=x.device)
    check(load().starkv_quantize_split(_ptr(x), dtype_code(x.dtype), rows, r, split_r, _ptr(up) if split_r else None,
                                       _ptr(s_up), _ptr(lo) if r4 else None, _ptr(s_lo), _stream()),
          "starkv_quantize_split")
    return up, s_up, lo, s_lo, r4


def set_test_hooks(wait_limit_ns: int = 0, skip_copy_unit: int = -1):
    """Test hooks of the device failure path (``starkv_set_test_hooks``); no
    arguments restore normal operation."""
    check(load().starkv_set_test_hooks(int(wait_limit_ns), int(skip_copy_unit)), "starkv_set_test_hooks")


def read_device_error(ws: Optional[torch.Tensor] = None, device="cuda") -> int:
    """Read and clear the kernels' device error word (synchronises)."""
    if ws is None:
        dev = torch.device(device)
        ws = _WORKSPACES.get((dev.type, dev.index))
        if ws is None:
            return 0
    code = C.c_int(0)
    check(load().starkv_read_device_error(_ptr(ws), C.byref(code), _stream()), "starkv_read_device_error")
    return int(code.value)


def prefill_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scaling: float,
                      out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
                      error_word: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Causal prompt attention (``starkv_prefill_attention``): q (B, Hq, T, 128),
    k / v (B, Hkv, T, 128), fp16 or bf16, any strides whose channel dimension is
    contiguous (e.g. ``x.view(B, T, H, 128).transpose(1, 2)``).  Returns (B, Hq, T, 128)
    in ``out_dtype`` (default: q's dtype), or writes ``out`` (any such strides)."""
    B, Hq, T, D = q.shape
    Hkv = k.shape[1]
    if D != 128 or k.shape != (B, Hkv, T, 128) or v.shape != (B, Hkv, T, 128):
        raise _lib.StarKVError("prefill_attention: q (B, Hq, T, 128), k / v (B, Hkv, T, 128)")
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise _lib.StarKVError("prefill_attention: q, k and v must share one dtype")
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.stride(3) != 1:
            raise _lib.StarKVError(f"prefill_attention: {name} channels must be contiguous")
    if out is None:
        out = torch.empty(B, Hq, T, 128, dtype=out_dtype or q.dtype, device=q.device)
    elif out.shape != (B, Hq, T, 128) or out.stride(3) != 1:
        raise _lib.StarKVError("prefill_attention: out must be (B, Hq, T, 128) with contiguous channels")
    a = _lib.PrefillArgs()
    a.q, a.k, a.v, a.out = _ptr(q), _ptr(k), _ptr(v), _ptr(out)
    for dst, t in ((a.q_strides, q), (a.k_strides, k), (a.v_strides, v), (a.out_strides, out)):
        dst[0], dst[1], dst[2] = t.stride(0), t.stride(1), t.stride(2)
    a.dtype, a.out_dtype = dtype_code(q.dtype), dtype_code(out.dtype)
    a.batch, a.num_q_heads, a.num_kv_heads, a.num_tokens = B, Hq, Hkv, T
    a.scaling = float(scaling)
    a.error_word = _ptr(error_word)
    check(load().starkv_prefill_attention(C.byref(a), _stream()), "starkv_prefill_attention")
    return out
