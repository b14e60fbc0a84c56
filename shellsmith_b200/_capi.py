"""ctypes binding of libshellcache.so, the C ABI every GPU call goes through.

The library is built in-tree (``shellsmith_b200/_build.py``). If it is missing
the import of a GPU entry point raises: there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().with_name("libshellcache.so")
_lib = None

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_F = ctypes.c_float

# name -> argument types, in the order of include/shellcache.h.
SIGNATURES = {
    "sc_version": [],
    "sc_last_error": [ctypes.c_char_p, _I],
    "sc_device_status": [ctypes.POINTER(ctypes.c_uint), _P],
    "sc_gdn_decode": [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P],
    "sc_gdn_decode_chained": [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P],
    "sc_gdn_decode_bf16": [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P],
    "sc_gdn_chunk_prefill": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I,
                             _I, _P],
    "sc_gdn_decode_fused": [_P, _P, _P, _P, _P, _P, _P, _P, _F, _P, _P, _P, _P, _P, _I, _I, _I,
                            _I, _P],
    "sc_gdn_decode_glue_workspace": [_I, _I, _I],
    "sc_gdn_decode_glue": [_P, _P, _P, _P, _P, _P, _P, _P, _F, _P, _P, _P, _P, _P, _P,
                           ctypes.c_size_t, _I, _I, _I, _I, _P],
    "sc_gdn_prefill_front": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I,
                             _I, _I, _I, _P],
    "sc_gdn_taps_store": [_P, _P, _P, _P, _P, _I, _I, _I, _P],
    "sc_gdn_sampler_gates": [_P, _P, _P, _P, _P, _P, _I64, _I, _P],
    "sc_gated_rmsnorm": [_P, _P, _P, _F, _P, _I64, _I, _P],
    "sc_exchange_put": [_P, ctypes.c_longlong, _P, _P, _P, ctypes.c_uint, _I, _P],
    "sc_exchange_wait": [_P, _I, _P, ctypes.c_uint, _P],
    "sc_exchange_wait_limited": [_P, _I, _P, ctypes.c_uint, ctypes.c_uint, _P],
    "sc_paged_decode_attention_exchange": [_P, _P, _I64, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I,
                                           _F, _P, _P, _P, _P, _P, _P, _P, ctypes.c_uint, _I,
                                           _P],
    "sc_attention_combine_exchange": [_P, _P, _P, ctypes.c_uint, _I, _I, _I, _P, _P, _P],
    "sc_kv_q8_block_bytes": [_I],
    "sc_kv_append_q8": [_P, _P, _P, _P, _I, _I, _I, _I, _I64, _P],
    "sc_kv_gather_q8": [_P, _P, _I, _I, _I, _I, _I64, _P, _P, _P],
    "sc_kv_copy_pages_q8": [_P, _P, _P, _I, _I, _I, _I, _I64, _P],
    "sc_paged_decode_attention_q8": [_P, _P, _I64, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I,
                                     _F, _P, _P, _P, _P, _P],
    "sc_kv_append": [_P, _P, _P, _P, _I, _I, _I, _I, _I64, _P],
    "sc_kv_gather": [_P, _P, _P, _P, _I, _I, _I, _I, _I64, _P],
    "sc_kv_copy_pages": [_P, _P, _P, _I, _I, _I, _I, _I64, _P],
    "sc_paged_decode_attention": [_P, _P, _I64, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I,
                                  _F, _P, _P, _P, _P, _P],
    "sc_attention_combine": [_P, _P, _I, _I, _I, _P, _P, _P],
    "sc_paged_decode_attention_packed": [_P, _P, _I64, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I,
                                         _F, _P, _P, _P, _P],
    "sc_attention_combine_packed": [_P, _I, _I, _I, _P, _P, _P],
    "sc_paged_decode_attention_fused": [_P, _P, _P, _P, _P, _I64, _P, _P, _P, _I, _I, _I, _I, _I,
                                        _I, _I, _I, _F, _P, _P, _P, _P, _P, _P, _I, _P],
    "sc_paged_decode_attention_noalloc": [_P, _P, _I64, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I,
                                          _F, _P, _P, _P],
}


RESTYPES = {"sc_gdn_decode_glue_workspace": ctypes.c_size_t}


class ShellcacheError(RuntimeError):
    """A nonzero status returned by the C ABI."""

    def __init__(self, name: str, code: int, text: str):
        super().__init__(f"{name} failed with status {code}: {text}")
        self.code = code


class DeviceFault(ShellcacheError):
    """A kernel set the device status word (bounded wait gave up, bad page index)."""


def library_path() -> Path:
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    """Load libshellcache.so once; raise if it was not built."""
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            raise ImportError(
                f"{_LIB_PATH} is missing: build it with `python -m shellsmith_b200._build` "
                "(the CUDA path has no CPU fallback)")
        handle = ctypes.CDLL(str(_LIB_PATH))
        for name, argtypes in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = argtypes
            fn.restype = RESTYPES.get(name, ctypes.c_int)
        _lib = handle
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    lib().sc_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def call(name: str, *args) -> None:
    """Call an entry point; raise ShellcacheError on a nonzero status."""
    code = getattr(lib(), name)(*args)
    if code != 0:
        raise ShellcacheError(name, code, last_error())


def device_status(stream: int = 0) -> int:
    """Read and clear the device status word (synchronises `stream`)."""
    word = ctypes.c_uint(0)
    call("sc_device_status", ctypes.byref(word), _P(stream))
    return int(word.value)


def check_device(stream: int = 0) -> None:
    """Raise DeviceFault if any kernel flagged a device-side fault since the last check."""
    word = device_status(stream)
    if word:
        reasons = []
        if word & 1:
            reasons.append("a bounded wait gave up")
        if word & 2:
            reasons.append("a page or slot index was outside the pool")
        raise DeviceFault("device status", 4, "; ".join(reasons) or f"word {word:#x}")
