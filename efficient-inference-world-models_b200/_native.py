"""ctypes binding of liboasis_b200.so (the C ABI declared in include/oasis_b200.h).

The library is the product: every call here forwards to a CUDA entry point and a
non-zero status becomes :class:`OasisError`.  There is no CPU fallback — if the
library is missing, importing :func:`lib` raises.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, Structure, c_char_p, c_float, c_int, c_longlong, c_size_t, c_uint8, c_void_p

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboasis_b200.so")

MAX_DEPTH = 16
MAX_FRAMES = 32
HIDDEN = 1024
TOKENS = 144
ADA_PER_SUB = 6 * HIDDEN

KV_BF16, KV_FP8, KV_INT4 = 0, 1, 2

STATUS_NAMES = {
    1: "invalid argument", 2: "alignment", 3: "workspace", 4: "CUDA error",
    5: "device timeout", 6: "unsupported",
}


class OasisError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"oasis_b200 error {status} ({STATUS_NAMES.get(status, '?')}): {message}")
        self.status = status


class SubWeights(Structure):
    _fields_ = [("qkv_w", c_void_p), ("out_w", c_void_p), ("out_b", c_void_p),
                ("fc1_w", c_void_p), ("fc1_b", c_void_p), ("fc2_w", c_void_p), ("fc2_b", c_void_p)]


class DiTWeights(Structure):
    _fields_ = [("depth", c_int),
                ("patch_w", c_void_p), ("patch_b", c_void_p),
                ("t_fc1_w", c_void_p), ("t_fc1_b", c_void_p),
                ("t_fc2_w", c_void_p), ("t_fc2_b", c_void_p),
                ("ada_w", c_void_p), ("ada_b", c_void_p),
                ("final_w", c_void_p), ("final_b", c_void_p),
                ("sub", SubWeights * (2 * MAX_DEPTH)),
                ("rope_spatial", c_void_p), ("rope_temporal", c_void_p)]


class KvTensor(Structure):
    """``oasis_kv_tensor_t``: the slot map and pools of the keys or of the values."""
    _fields_ = [("n_bf16", c_int), ("n_fp8", c_int), ("n_int4", c_int),
                ("slot_kind", c_uint8 * MAX_FRAMES), ("slot_index", c_uint8 * MAX_FRAMES),
                ("bf16", c_void_p), ("fp8", c_void_p), ("fp8_scale", c_void_p),
                ("int4", c_void_p), ("i4_scale", c_void_p), ("i4_zero", c_void_p)]


class KvCache(Structure):
    """``oasis_kv_cache_t``: ``k`` the keys, ``v`` the values."""
    _fields_ = [("batch", c_int), ("layers", c_int), ("n_slots", c_int),
                ("k", KvTensor), ("v", KvTensor)]


KV_KEYS, KV_VALUES = 1, 2

VAE_MAX_DEPTH = 12
VAE_PRED_LD = 1216


class VaeBlock(Structure):
    """``oasis_vae_block_t``: one pre-norm block of the latent decoder."""
    _fields_ = [("ln1_shift", c_void_p), ("ln1_scale", c_void_p), ("qkv_w", c_void_p),
                ("proj_w", c_void_p), ("proj_b", c_void_p), ("ln2_shift", c_void_p),
                ("ln2_scale", c_void_p), ("fc1_w", c_void_p), ("fc1_b", c_void_p),
                ("fc2_w", c_void_p), ("fc2_b", c_void_p)]


class VaeWeights(Structure):
    """``oasis_vae_weights_t``."""
    _fields_ = [("depth", c_int), ("post_w", c_void_p), ("post_b", c_void_p),
                ("blk", VaeBlock * VAE_MAX_DEPTH), ("norm_shift", c_void_p), ("norm_scale", c_void_p),
                ("pred_w", c_void_p), ("pred_b", c_void_p), ("rope", c_void_p), ("ones", c_void_p)]


# name -> (restype, argtypes); every symbol include/oasis_b200.h declares
SIGNATURES = {
    "oasis_last_error": (c_char_p, []),
    "oasis_version": (c_char_p, []),
    "oasis_check_device_error": (c_int, []),
    "oasis_selftest_bounded_wait": (c_int, [c_void_p]),
    "oasis_plan_workspace_size": (c_size_t, [c_int, c_int, c_int]),
    "oasis_plan_create": (c_int, [POINTER(DiTWeights), c_int, c_int, c_void_p, c_size_t,
                                  POINTER(c_void_p)]),
    "oasis_plan_destroy": (None, [c_void_p]),
    "oasis_dit_forward": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                  POINTER(KvCache), c_void_p]),
    "oasis_dit_forward_cached": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                         POINTER(KvCache), c_int, c_void_p]),
    "oasis_dit_forward_noalloc": (c_int, [POINTER(DiTWeights), c_int, c_int, c_void_p, c_void_p,
                                          c_void_p, c_void_p, c_void_p]),
    "oasis_plan_set_timing": (c_int, [c_void_p, c_int]),
    "oasis_plan_get_timing": (c_int, [c_void_p, POINTER(c_float), POINTER(c_int), c_int]),
    "oasis_gemm_bf16": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                c_int, c_int, c_int, c_int, c_void_p]),
    "oasis_attn_spatial": (c_int, [c_void_p, c_void_p, c_int, c_void_p]),
    "oasis_attn_temporal": (c_int, [c_void_p, POINTER(KvCache), c_int, c_void_p, c_int, c_int,
                                    c_int, c_int, c_int, c_void_p]),
    "oasis_kv_store": (c_int, [c_void_p, c_int, c_int, c_int, POINTER(KvCache), c_int, c_int,
                               c_int, c_int, c_void_p]),
    "oasis_kv_migrate": (c_int, [POINTER(KvCache), c_int, c_int, c_int, c_void_p]),
    "oasis_kv_load": (c_int, [POINTER(KvCache), c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "oasis_dpmpp2m_update": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_longlong,
                                     c_longlong, c_float, c_float, c_int, c_void_p]),
    "oasis_ab_update": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_longlong,
                                c_float, c_float, c_float, c_float, c_void_p]),
    "oasis_vae_workspace_size": (c_size_t, [c_int, c_int]),
    "oasis_vae_plan_create": (c_int, [POINTER(VaeWeights), c_int, c_void_p, c_size_t, POINTER(c_void_p)]),
    "oasis_vae_plan_destroy": (None, [c_void_p]),
    "oasis_vae_decode": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p]),
}

_LIB = None


def lib() -> ctypes.CDLL:
    """Load liboasis_b200.so (built by ``build.py``); raises if it is absent."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def check(status: int) -> None:
    if status != 0:
        msg = lib().oasis_last_error().decode(errors="replace")
        raise OasisError(status, msg)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))


def version() -> str:
    return lib().oasis_version().decode()
