"""ctypes binding of ``libq35b200.so`` (the C ABI in ``include/q35b200.h``).

The library is loaded from the package directory, where
``qwen3_5_vl_cuda_custom_b200.build`` puts it.  There is no fallback: if the
library is missing or a call returns a non-zero status, a RuntimeError names
the entry point, the status and the library's detail message.
"""
from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_int64, c_void_p, c_char_p, POINTER
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libq35b200.so"

_i32p = POINTER(ctypes.c_int32)

# name -> (restype, argtypes).  Pointers are passed as c_void_p (ints).
_SIGS = {
    "q35_status_string": (c_char_p, [c_int]),
    "q35_last_error_message": (c_char_p, []),
    "q35_device_error_check": (c_int, [_i32p]),
    "q35_version": (c_char_p, []),
    "q35_set_sm_limit": (c_int, [c_int]),
    "q35_launch_count": (c_int64, []),
    "q35_embedding_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p]),
    "q35_vision_qkv_rope_pad": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                                        c_int, c_int, c_int, c_void_p]),
    "q35_unpad_heads": (c_int, [c_void_p, c_void_p, c_int64, c_int, c_int, c_int, c_void_p]),
    "q35_selftest_wait_timeout": (c_int, [c_int64, c_void_p]),
    "q35_rmsnorm_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_float, c_void_p]),
    "q35_qknorm_mrope_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, _i32p, c_int,
                                     c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int, c_int,
                                     c_int, c_float, c_void_p]),
    "q35_qkv_proj_norm_rope": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, _i32p,
                                       c_int, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int,
                                       c_int, c_int, c_float, c_void_p, c_void_p]),
    "q35_mrope_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, _i32p, c_int, c_int64, c_int,
                              c_int64, c_int, c_void_p]),
    "q35_router_topk_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                    c_void_p, c_int64, c_int, c_int, c_int, c_int, c_void_p,
                                    c_void_p]),
    "q35_router_workspace": (c_int64, [c_int64, c_int, c_int]),
    "q35_router_split_weights": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "q35_router_logits_tc": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int, c_int,
                                     c_void_p]),
    "q35_softmax_fwd": (c_int, [c_void_p, c_void_p, c_int64, c_int, c_void_p]),
    "q35_topk_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int, c_void_p]),
    "q35_moe_permute_workspace": (c_int64, [c_int64, c_int]),
    "q35_moe_permute": (c_int, [c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                c_void_p, c_void_p, c_void_p, c_void_p]),
    "q35_router_fused_supported": (c_int, [c_int64, c_int, c_int, c_int]),
    "q35_router_topk_fused": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                      c_void_p, c_int64, c_int, c_int, c_int, c_int, c_void_p]),
    "q35_moe_permute_counted": (c_int, [c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p,
                                        c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "q35_moe_permute_slabs": (c_int, [c_void_p, c_int, c_int64, c_void_p, c_int, c_int, c_void_p,
                                      c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "q35_ep_window_bytes": (c_int64, [c_int, c_int64, c_int64, c_int]),
    "q35_ep_window_offsets": (c_int, [c_int, c_int64, c_int64, c_int, POINTER(c_int64)]),
    "q35_ep_window_alloc": (c_int, [c_int, c_int64, c_int64, c_int, POINTER(c_void_p)]),
    "q35_ep_window_free": (c_int, [c_void_p]),
    "q35_ep_ipc_handle": (c_int, [c_void_p, c_void_p]),
    "q35_ep_ipc_open": (c_int, [c_void_p, POINTER(c_void_p)]),
    "q35_ep_ipc_close": (c_int, [c_void_p]),
    "q35_ep_set_peers": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int, c_void_p]),
    "q35_ep_dispatch": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int64, c_int, c_int,
                                c_int, c_int64, c_void_p, c_void_p, c_void_p, c_void_p]),
    "q35_ep_wait": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int, c_int, c_int64, c_void_p]),
    "q35_ep_return": (c_int, [c_void_p, c_void_p, c_int64, c_int, c_int64, c_int, c_int, c_void_p,
                              c_void_p]),
    "q35_moe_permute_noalloc_max_workspace": (c_int64, []),
    "q35_moe_permute_noalloc": (c_int, [c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                        c_void_p, c_void_p, c_void_p]),
    "q35_ep_scatter": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int64, c_int, c_int,
                               c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p]),
    "q35_gather_rows": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_int64, c_void_p]),
    "q35_gemm_bf16": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64,
                              c_int64, c_void_p]),
    "q35_grouped_gemm_gateup_swiglu": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                               c_int, c_int64, c_int, c_int, c_int, c_void_p]),
    "q35_attn_prefill_cache_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                                           c_int, c_int, c_int64, c_int64, c_int64, c_int, c_float,
                                           c_int, c_void_p]),
    "q35_attn_decode_cache_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int,
                                          c_int64, c_int64, c_int64, c_int, c_float, c_void_p,
                                          c_void_p]),
    "q35_kv_append": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int64, c_int,
                              c_int64, c_int64, c_void_p]),
    "q35_layernorm_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_float,
                                  c_void_p]),
    "q35_gelu_tanh_fwd": (c_int, [c_void_p, c_void_p, c_int64, c_void_p]),
    "q35_rope_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int64, c_int,
                             c_int, c_int, c_void_p]),
    "q35_conv3d_patch_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                     c_void_p]),
    "q35_gemm_bf16_splitk": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int64,
                                     c_int64, c_int64, c_int, c_void_p, c_void_p]),
    "q35_grouped_gemm_down": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                                      c_int64, c_int, c_int, c_int, c_void_p]),
    "q35_pack_b_tiles": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p]),
    "q35_moe_combine": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int64,
                                c_int, c_int64, c_void_p]),
    "q35_rmsnorm_f32in_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_float,
                                      c_void_p]),
    "q35_gemm_bf16_f32out": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                                     c_int64, c_int64, c_void_p]),
    "q35_index_add": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int,
                              c_void_p]),
    "q35_swiglu_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "q35_residual_add_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "q35_attn_prefill_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                                     c_int, c_int, c_int64, c_int64, c_int, c_float, c_int,
                                     c_void_p]),
    "q35_attn_decode_workspace": (c_int64, [c_int64, c_int, c_int64, c_int64, c_int]),
    "q35_attn_decode_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int,
                                    c_int64, c_int64, c_int, c_float, c_void_p, c_void_p]),
}

EXPORTED = tuple(_SIGS)

_lib = None


def load() -> ctypes.CDLL:
    """Loads the kernel library once; raises ImportError when it was never built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH.name} is not built: run `python -m qwen3_5_vl_cuda_custom_b200.build`")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def call(name: str, *args) -> None:
    """Calls a status-returning entry point and raises on a non-zero status."""
    lib = load()
    st = getattr(lib, name)(*args)
    if st != 0:
        msg = lib.q35_last_error_message().decode(errors="replace")
        what = lib.q35_status_string(st).decode()
        raise RuntimeError(f"{name}: {what} ({st}): {msg}")


def query(name: str, *args):
    """Calls a value-returning entry point (workspace sizes, strings)."""
    return getattr(load(), name)(*args)


def device_error_check() -> tuple[int, int, int, int]:
    """Synchronises the current device and raises if a kernel recorded an error."""
    info = (ctypes.c_int32 * 4)()
    lib = load()
    st = lib.q35_device_error_check(info)
    if st != 0:
        msg = lib.q35_last_error_message().decode(errors="replace")
        raise RuntimeError(f"device error: {msg}")
    return tuple(info)


def sections_arg(sections) -> ctypes.Array:
    arr = (ctypes.c_int32 * 3)(*[int(s) for s in sections])
    return arr
