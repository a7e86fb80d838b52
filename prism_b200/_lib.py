"""ctypes binding of the C ABI in include/prism_bsa.h (libprism_bsa.so).

The library is built in-tree (prism_b200/libprism_bsa.so) by prism_b200.build.
There is no fallback: if the library cannot be loaded every op raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_F = ctypes.c_float
_D = ctypes.c_double
_SZ = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/prism_bsa.h
SIGNATURES = {
    "prism_last_error": (ctypes.c_char_p, []),
    "prism_abi_version": (_I, []),
    "prism_device_status": (_I, []),
    "prism_test_fwd_withheld_load": (_I, [_P, _P, _P, _I64, _I, _F, _P, _P, _P, _P, ctypes.c_uint64, _P]),
    "prism_token_norms": (_I, [_P, _I64, _I, _P, _P]),
    "prism_gemm_bf16": (_I, [_P, _I64, _I, _P, _I64, _I, _I, _I, _I, _P, _P, _I64, _I, _P]),
    "prism_zone_stats_workspace_bytes": (_SZ, [_I, _I, _I, _I]),
    "prism_zone_stats": (_I, [_P, _I, _I64, _I64, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P]),
    "prism_shape_select": (_I, [_P, _P, _P, _I, _I, _I, _I, _F, _F, _F, _P, _P, _P, _P]),
    "prism_build_layout": (_I, [_P, _I, _I, _I, _P, _P, _P, _P, _P, _P]),
    "prism_tile_valid": (_I, [_P, _I64, _P, _I, _I, _I, _I, _I, _I, _P, _P, _P]),
    "prism_gather_rows": (_I, [_P, _I64, _I64, _I, _I, _I, _I, _I, _I, _I, _I, _P, _I64, _P, _I64, _P]),
    "prism_scatter_rows": (_I, [_P, _I64, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _I64, _I64, _P]),
    "prism_copy_rows": (_I, [_P, _I64, _I64, _P, _I64, _I64, _I64, _I64, _I64, _P]),
    "prism_block_select_workspace_bytes": (_SZ, [_I, _I64, _I]),
    "prism_block_select": (_I, [_P, _P, _I, _I64, _I, _P, _P, _P, _I, _D, _D, _P, _P, _P, _P]),
    "prism_uniform_layout": (_I, [_I, _I, _I, _I, _I, _I, _I64, _P, _P, _P]),
    "prism_block_select_uniform_workspace_bytes": (_SZ, [_I, _I64, _I64, _I]),
    "prism_block_select_uniform": (_I, [_P, _P, _I, _I64, _I64, _I, _I64, _I64, _I, _I, _P, _P, _P, _P, _I, _D, _D, _P, _P, _P, _P]),
    "prism_gather_values": (_I, [_P, _I, _I, _I, _I, _I, _I, _P, _I64, _P, _P]),
    "prism_variance_density": (_I, [_P, _I, _I64, _I, _I64, _I, _I, _I, _P, _P, _P]),
    "prism_audio_saliency": (_I, [_P, _I64, _I, _P, _P, _P]),
    "prism_audio_pool_weights": (_I, [_P, _I64, _I, _P, _F, _P, _P]),
    "prism_guidance_scale": (_I, [_I64, _P, _F, _P, _P, _F, _P, _P, _P]),
    "prism_pool_chunks": (_I, [_P, _I, _I64, _I, _I64, _I, _P, _P, _P, _P]),
    "prism_chunk_scores": (_I, [_P, _P, _I, _I, _I, _I, _P, _P]),
    "prism_bsa_fwd_keybias": (_I, [_P, _P, _P, _I, _I64, _I64, _I, _F, _P, _P, _P, _P, _P, _P, _P]),
    "prism_correction_stats": (_I, [_P, _I, _I, _I, _I, _I, _P, _I64, _I64, _P, _F, _P, _P, _P, _P, _P]),
    "prism_taylor_prep": (_I, [_P, _P, _P, _I, _I64, _I, _I, _I, _I64, _P, _P, _P]),
    "prism_key_log_bias": (_I, [_P, _I, _I, _I, _F, _P, _P]),
    "prism_rows_to_bf16": (_I, [_P, _I, _I, _I, _I, _P, _P]),
    "prism_taylor_merge": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I64, _I64, _I, _I, _P, _P]),
    "prism_rectified_contract": (_I, [_P, _P, _I, _I, _I, _I, _P, _P]),
    "prism_rectified_apply": (_I, [_P, _P, _P, _P, _I, _I64, _I64, _I, _I, _P, _P]),
    "prism_norm_rope_pack": (_I, [_P, _I64, _I64, _I64, _I, _I, _I, _I, _P, _F, _P, _I, _P, _P, _P]),
    "prism_norm_rope_pack_bwd_workspace_bytes": (_SZ, [_I64, _I, _I]),
    "prism_norm_rope_pack_bwd": (_I, [_P, _P, _I64, _I64, _I64, _I, _I, _I, _I, _P, _P, _P, _I, _P, _I64,
                                      _P, _P, _P]),
    "prism_bsa_fwd_qk": (_I, [_P, _P, _P, _I, _I64, _I64, _I, _F, _P, _P, _P, _P, _P, _P]),
    "prism_bsa_bwd_qk": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I64, _I64, _I, _F, _P, _P, _P, _P, _P, _P, _P, _P]),
    "prism_bsa_fwd": (_I, [_P, _P, _P, _I, _I64, _I, _F, _P, _P, _P, _P, _P, _P]),
    "prism_bsa_bwd_workspace_bytes": (_SZ, [_I, _I64]),
    "prism_bsa_bwd": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I64, _I, _F, _P, _P, _P, _P, _P, _P, _P, _P]),
    "prism_bsa_bwd_delta": (_I, [_P, _P, _P, _I, _I64, _I, _P, _P]),
    "prism_bsa_bwd_dkdv": (_I, [_P, _P, _P, _P, _P, _P, _I, _I64, _I, _F, _P, _P, _P, _P, _P]),
    "prism_bsa_bwd_dq": (_I, [_P, _P, _P, _P, _P, _P, _I, _I64, _I, _F, _P, _P, _P, _P]),
    "prism_bsa_bwd_noalloc": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I64, _I, _F, _P, _P, _P, _P, _P, _P, _P]),
}

# kernels launched per entry point (the bench's gpu_launches count)
KERNELS = {
    "prism_token_norms": 1, "prism_zone_stats": 2, "prism_shape_select": 1,
    "prism_build_layout": 2, "prism_tile_valid": 1, "prism_gather_rows": 1,
    "prism_scatter_rows": 1, "prism_copy_rows": 1, "prism_block_select": 4, "prism_bsa_fwd": 1, "prism_bsa_bwd": 3,
    "prism_bsa_bwd_delta": 1, "prism_bsa_bwd_dkdv": 1, "prism_bsa_bwd_dq": 1,
    "prism_bsa_bwd_noalloc": 3, "prism_uniform_layout": 1, "prism_block_select_uniform": 4,
    "prism_bsa_fwd_qk": 1, "prism_bsa_bwd_qk": 3, "prism_gather_values": 1,
    "prism_variance_density": 2, "prism_audio_saliency": 2, "prism_audio_pool_weights": 1,
    "prism_guidance_scale": 1, "prism_pool_chunks": 1, "prism_chunk_scores": 1,
    "prism_bsa_fwd_keybias": 1, "prism_correction_stats": 1, "prism_taylor_prep": 1,
    "prism_key_log_bias": 1, "prism_rows_to_bf16": 1, "prism_taylor_merge": 1,
    "prism_rectified_apply": 1, "prism_rectified_contract": 1, "prism_norm_rope_pack": 1,
    "prism_gemm_bf16": 1, "prism_norm_rope_pack_bwd": 4,
}
launch_count = 0

_lock = threading.Lock()
_lib = None


class PrismError(RuntimeError):
    pass


def lib_path() -> str:
    return _build.LIB


def load(build_if_missing: bool = True):
    """Load libprism_bsa.so (building it first if it is absent and nvcc exists)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = _build.LIB
        if not os.path.exists(path):
            if not build_if_missing:
                raise PrismError(f"{path} is missing; run `python -m prism_b200.build`")
            _build.build()
        L = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
        return L


def call(name: str, *args):
    """Invoke an entry point; raise PrismError with the library's message on failure."""
    global launch_count
    L = load()
    rc = getattr(L, name)(*args)
    launch_count += KERNELS.get(name, 0)
    if rc != 0:
        msg = L.prism_last_error().decode(errors="replace")
        if "Either sparsity or cdf_threshold" in msg or "unknown dynamic-block method" in msg:
            raise ValueError(msg)
        raise PrismError(f"{name} failed ({rc}): {msg}")
    return rc


def query(name: str, *args) -> int:
    return int(getattr(load(), name)(*args))
