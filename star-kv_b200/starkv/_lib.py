"""ctypes binding of ``libstarkv.so`` (the C ABI declared in ``include/starkv.h``).

The shared library is built in-tree by ``starkv.build`` (nvcc, sm_100a).  There
is no fallback: if the library is missing every op raises.
"""

from __future__ import annotations

import ctypes as C
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libstarkv.so")

ABI_VERSION = 2
MAX_KV_HEADS = 64
MAX_V_BLOCKS = 32

F32, F16, BF16 = 0, 1, 2

STATUS = {0: "OK", 1: "INVALID", 2: "UNSUPPORTED", 3: "LAUNCH", 4: "WORKSPACE", 5: "DEVICE"}


class Layout(C.Structure):
    """Mirror of ``starkv_layout``."""

    _fields_ = [
        ("abi_version", C.c_int32), ("batch", C.c_int32), ("num_q_heads", C.c_int32),
        ("num_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("num_v_blocks", C.c_int32),
        ("capacity", C.c_int32), ("quantized", C.c_int32), ("latent_dtype", C.c_int32),
        ("k_rank_total", C.c_int32), ("v_rank_total", C.c_int32), ("k_tiled", C.c_int32),
        ("k_rank", C.c_int32 * MAX_KV_HEADS), ("k_col", C.c_int32 * MAX_KV_HEADS),
        ("k_offset", C.c_int64 * MAX_KV_HEADS), ("k_batch_stride", C.c_int64 * MAX_KV_HEADS),
        ("v_rank", C.c_int32 * MAX_V_BLOCKS), ("v_col", C.c_int32 * MAX_V_BLOCKS),
        ("v_first_kv", C.c_int32 * MAX_V_BLOCKS), ("v_num_kv", C.c_int32 * MAX_V_BLOCKS),
    ]


class DecodeArgs(C.Structure):
    """Mirror of ``starkv_decode_args``."""

    _fields_ = [
        ("q", C.c_void_p), ("q_dtype", C.c_int32), ("w_dtype", C.c_int32),
        ("k_u", C.c_void_p), ("v_u", C.c_void_p), ("inv_freq", C.c_void_p), ("mask", C.c_void_p),
        ("scaling", C.c_float), ("num_tokens", C.c_int32),
        ("k_cache", C.c_void_p), ("k_scales", C.c_void_p), ("v_cache", C.c_void_p), ("v_params", C.c_void_p),
        ("out", C.c_void_p), ("out_dtype", C.c_int32),
        ("num_splits", C.c_int32),
        ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t),
        ("events", C.POINTER(C.c_void_p)),
    ]


class PrefillArgs(C.Structure):
    """Mirror of ``starkv_prefill_args``."""

    _fields_ = [
        ("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p),
        ("q_strides", C.c_int64 * 3), ("k_strides", C.c_int64 * 3), ("v_strides", C.c_int64 * 3),
        ("dtype", C.c_int32), ("batch", C.c_int32), ("num_q_heads", C.c_int32), ("num_kv_heads", C.c_int32),
        ("num_tokens", C.c_int32), ("scaling", C.c_float),
        ("out", C.c_void_p), ("out_dtype", C.c_int32), ("out_strides", C.c_int64 * 3),
        ("error_word", C.c_void_p),
    ]


# (name, restype, argtypes) of every exported symbol; tests check the header declares exactly these.
SIGNATURES = [
    ("starkv_layout_size", C.c_size_t, []),
    ("starkv_validate_layout", C.c_int, [C.POINTER(Layout)]),
    ("starkv_quantize_prefill", C.c_int, [C.POINTER(Layout), C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p,
                                          C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    ("starkv_append", C.c_int, [C.POINTER(Layout), C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_void_p,
                                C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    ("starkv_project_append", C.c_int, [C.POINTER(Layout), C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_int32,
                                        C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                        C.c_void_p]),
    ("starkv_decode_workspace_size", C.c_int, [C.POINTER(Layout), C.c_int32, C.c_int32, C.POINTER(C.c_size_t)]),
    ("starkv_auto_splits", C.c_int32, [C.POINTER(Layout), C.c_int32]),
    ("starkv_decode_attention", C.c_int, [C.POINTER(Layout), C.POINTER(DecodeArgs), C.c_void_p]),
    ("starkv_k_logits", C.c_int, [C.POINTER(Layout), C.POINTER(DecodeArgs), C.c_void_p, C.c_void_p]),
    ("starkv_v_latent", C.c_int, [C.POINTER(Layout), C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p,
                                  C.c_void_p]),
    ("starkv_set_test_hooks", C.c_int, [C.c_int64, C.c_int32]),
    ("starkv_quantize_split", C.c_int, [C.c_void_p, C.c_int32, C.c_int64, C.c_int32, C.c_int32, C.c_void_p,
                                        C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    ("starkv_decode_attention_static", C.c_int, [C.POINTER(Layout), C.POINTER(DecodeArgs), C.c_void_p]),
    ("starkv_static_scratch_bytes", C.c_size_t, []),
    ("starkv_static_read_device_error", C.c_int, [C.POINTER(C.c_int), C.c_void_p]),
    ("starkv_read_device_error", C.c_int, [C.c_void_p, C.POINTER(C.c_int), C.c_void_p]),
    ("starkv_prefill_attention", C.c_int, [C.POINTER(PrefillArgs), C.c_void_p]),
    ("starkv_last_error", C.c_char_p, []),
]

_lib = None


class StarKVError(RuntimeError):
    pass


def load(path: str = LIB_PATH):
    """Load (once) and return the bound library; raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise StarKVError(f"libstarkv.so not found at {path}; build it with starkv.build.build()")
    lib = C.CDLL(path)
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.starkv_layout_size() != C.sizeof(Layout):
        raise StarKVError("starkv_layout size mismatch between libstarkv.so and the Python binding")
    _lib = lib
    return lib


def check(rc: int, what: str):
    if rc != 0:
        msg = load().starkv_last_error().decode(errors="replace")
        raise StarKVError(f"{what} failed: {STATUS.get(rc, rc)}: {msg}")
