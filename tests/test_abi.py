"""libstarkv.so loads on a CPU-only machine, exports exactly what include/starkv.h
declares, and validates layouts on the host (no CUDA calls)."""

import ctypes as C
import os
import re

import pytest

from conftest import ROOT
from starkv import _lib


def header_functions():
    src = open(os.path.join(ROOT, "include", "starkv.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return set(re.findall(r"\b(starkv_\w+)\s*\(", src))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = header_functions()
    bound = {name for name, _, _ in _lib.SIGNATURES}
    assert declared == bound, declared ^ bound
    for name in declared:
        assert hasattr(lib, name), name


def test_layout_abi_size():
    lib = _lib.load()
    assert lib.starkv_layout_size() == C.sizeof(_lib.Layout)


def test_layout_validation_host_only():
    import torch
    from starkv import ops
    lay = ops.make_layout(2, 8, 8, [16, 32, 96, 48, 16, 16, 64, 80], [64, 192], [4, 4], 300, True, torch.float16)
    assert lay.k_rank_total == 368 and lay.v_rank_total == 256
    lib = _lib.load()
    bad = ops.make_layout(2, 8, 8, [16] * 8, [64, 64], [4, 4], 10, True, torch.float16)
    bad.k_rank[0] = 24                                               # not a multiple of 16
    assert lib.starkv_validate_layout(C.byref(bad)) == 2
    bad.k_rank[0] = 16
    bad.v_num_kv[1] = 3                                              # blocks do not cover the heads
    assert lib.starkv_validate_layout(C.byref(bad)) == 1
    with pytest.raises(_lib.StarKVError):
        ops.make_layout(2, 8, 8, [256] * 8, [64, 64], [4, 4], 10, True, torch.float16)
    with pytest.raises(_lib.StarKVError):                            # 64 q heads in one V block
        ops.make_layout(1, 64, 8, [32] * 8, [64], [8], 10, True, torch.float16)
    with pytest.raises(_lib.StarKVError):                            # V block rank above 1024
        ops.make_layout(1, 8, 8, [32] * 8, [1056], [8], 10, True, torch.float16)


def test_no_cpu_path():
    """The ops refuse CPU tensors instead of computing on the host."""
    import torch
    from starkv import ops
    lay = ops.make_layout(1, 4, 4, [16] * 4, [64], [4], 8, True, torch.float16)
    with pytest.raises(_lib.StarKVError):
        ops._ptr(torch.zeros(4))


def test_tiled_k_layout_host_rules():
    """The default cache layout tiles K by 128 slots (capacity rounded up); a
    tiled layout whose capacity is not a multiple of 128 is rejected, the
    reference's row-major (B, Hkv, L, r) layout accepts any capacity."""
    import torch
    from starkv import ops
    lib = _lib.load()
    lay = ops.make_layout(2, 8, 8, [16, 32, 96, 48, 16, 16, 64, 80], [64, 192], [4, 4], 300, True, torch.float16)
    assert lay.k_tiled == 1 and lay.capacity == 384
    assert lib.starkv_validate_layout(C.byref(lay)) == 0
    lay.capacity = 300
    assert lib.starkv_validate_layout(C.byref(lay)) == 1
    rm = ops.make_layout(1, 4, 4, [32] * 4, [64], [4], 300, False, torch.float16,
                         k_offsets=[h * 300 * 32 for h in range(4)], k_batch_strides=[4 * 300 * 32] * 4)
    assert rm.k_tiled == 0 and rm.capacity == 300
    assert lib.starkv_validate_layout(C.byref(rm)) == 0


def test_tiled_k_head_view_inverts_the_tiling():
    """LatentCache.k_head de-tiles: element (b, slot, c) of the tiled layout sits at
    k_offset + b*stride + (slot//128)*128*r + (c//n)*128*n + (slot%128)*n + c%n."""
    import torch
    from starkv import ops
    lay = ops.make_layout(2, 2, 2, [48, 16], [64], [2], 200, True, torch.float16)
    cache = ops.LatentCache.__new__(ops.LatentCache)
    cache.layout = lay
    n_el = lay.batch * lay.capacity * lay.k_rank_total
    cache.k_cache = torch.arange(n_el, dtype=torch.int32)     # 4-byte elements: 4 per 16-byte chunk
    n = 4
    for h, r in enumerate([48, 16]):
        view = cache.k_head(h)
        for (b, slot, c) in [(0, 0, 0), (1, 130, r - 1), (0, 255, 17 % r), (1, 5, 6), (1, 255, r - 2)]:
            idx = (lay.k_offset[h] + b * lay.k_batch_stride[h] + (slot // 128) * 128 * r + (c // n) * 128 * n
                   + (slot % 128) * n + c % n)
            assert int(view[b, slot, c]) == idx
