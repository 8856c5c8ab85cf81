"""ctypes binding of libhexgen2_b200.so (the C ABI declared in include/hexgen2_b200.h).

There is no fallback: if the library is missing or cannot be loaded, importing the kernel
ops raises. Build it with `python -m hexgen2_b200.build`.
"""
from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_int64, c_size_t, c_void_p, c_char_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libhexgen2_b200.so")

HX_OK, HX_ERR_INVALID, HX_ERR_UNSUPPORTED, HX_ERR_CUDA, HX_ERR_DEVICE = range(5)
HX_F32, HX_F16, HX_BF16 = 0, 1, 2
HX_EPI_NONE, HX_EPI_RESIDUAL, HX_EPI_SWIGLU, HX_EPI_QKV_ROTARY = 0, 1, 2, 3

_SIGNATURES = {
    "hx_abi_version": (c_int, []),
    "hx_last_error": (c_char_p, []),
    "hx_device_error": (c_int, [c_int]),
    "hx_sm_count": (c_int, []),
    "hx_embedding": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int64, c_void_p,
                             c_int, c_void_p]),
    "hx_embed_rmsnorm": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_float,
                                 c_void_p, c_void_p, c_int, c_void_p]),
    "hx_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64,
                           c_int64, c_int64, c_float, c_int, c_void_p]),
    "hx_rotary_cache_write": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64,
                                      c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p,
                                      c_void_p, c_int64, c_int64, c_int64, c_int64, c_int,
                                      c_void_p]),
    "hx_gemm": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64,
                        c_int64, c_int64, c_int, c_void_p, c_int64, c_void_p, c_size_t, c_int,
                        c_void_p]),
    "hx_gemm_workspace": (c_size_t, [c_int64, c_int64, c_int64, c_int, c_int]),
    "hx_gemm_kernel_kind": (c_int, [c_int64, c_int64, c_int64, c_int]),
    "hx_gemm_qkv_rotary": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64,
                                   c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_int64,
                                   c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64,
                                   c_void_p, c_size_t, c_int, c_void_p]),
    "hx_gemm_qkv_rotary_varlen": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                          c_void_p, c_void_p, c_void_p, c_int64, c_int64,
                                          c_int64, c_int64, c_void_p, c_void_p, c_int64,
                                          c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64,
                                          c_void_p, c_size_t, c_int, c_void_p]),
    "hx_prefill_attention": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p,
                                     c_int64, c_int64, c_int64, c_int64, c_int64, c_int, c_float,
                                     c_void_p, c_int, c_void_p]),
    "hx_prefill_attention_varlen": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                            c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                                            c_int64, c_int64, c_int64, c_int64, c_int64, c_int,
                                            c_float, c_void_p, c_int, c_void_p]),
    "hx_decode_attention": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_int64,
                                    c_int64, c_int64, c_int64, c_int64, c_float, c_void_p,
                                    c_void_p, c_size_t, c_int, c_void_p]),
    "hx_decode_attention_workspace": (c_size_t, [c_int64, c_int64, c_int64, c_int64]),
    "hx_decode_attention_noalloc": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_int64,
                                            c_int64, c_int64, c_int64, c_int64, c_float, c_void_p,
                                            c_int, c_void_p]),
    "hx_argmax": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int, c_void_p]),
    "hx_kv_pack": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64,
                           c_int64, c_int64, c_void_p, c_void_p]),
    "hx_kv_unpack": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                             c_int64, c_int64, c_int64, c_void_p]),
    "hx_enable_peer_access": (c_int, [c_int]),
    "hx_ipc_get_handle": (c_int, [c_void_p, c_void_p]),
    "hx_ipc_open_handle": (c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    "hx_ipc_close_handle": (c_int, [c_void_p]),
    "hx_mem_range": (c_int, [c_void_p, ctypes.POINTER(c_void_p), ctypes.POINTER(c_size_t)]),
    "hx_peer_copy": (c_int, [c_void_p, c_int, c_void_p, c_int, c_size_t, c_void_p]),
}


class KernelError(RuntimeError):
    """A CUDA-side failure reported by the hexgen2_b200 library."""


_lib = None


def lib() -> ctypes.CDLL:
    """Loads the library once; raises ImportError if it is missing."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is not built; run `python -m hexgen2_b200.build`")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (restype, argtypes) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = handle
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def check(status: int, what: str = "") -> None:
    """Maps an hx_status to the reference's exception conventions."""
    if status == HX_OK:
        return
    msg = (lib().hx_last_error() or b"").decode(errors="replace")
    text = f"{what}: {msg}" if what else msg
    if status == HX_ERR_INVALID:
        raise ValueError(text)
    if status == HX_ERR_UNSUPPORTED:
        raise NotImplementedError(text)
    raise KernelError(f"{text} (status {status})")
