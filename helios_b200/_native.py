"""ctypes binding of ``libhelios_b200.so`` (the C ABI in ``include/helios_b200.h``).

The library is built in-tree by ``helios_b200.build`` (nvcc, sm_100a). There is
no fallback: if the library is missing or fails to load, every op raises.
Loading does not touch the GPU, so the symbol table can be checked on a CPU host.
"""

from __future__ import annotations

import ctypes
import re
from ctypes import c_float, c_int, c_int32, c_int64, c_size_t, c_uint32, c_void_p
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "_lib" / "libhelios_b200.so"
HEADER = PKG.parent / "include" / "helios_b200.h"

HB_OK = 0
HB_ERR_INVALID = -1
HB_ERR_UNSUPPORTED = -2
HB_ERR_CUDA = -3

STATUS_BITS = {
    1 << 0: "wait timeout",
    1 << 1: "KV write slot outside the pool",
    1 << 2: "RoPE position outside the tables",
    1 << 3: "page index outside the pool",
    1 << 4: "token id outside the vocabulary",
    1 << 5: "row index outside its tensor",
    1 << 6: "prefix index full",
}

P = c_void_p
I32 = c_int32
I64 = c_int64
F32 = c_float

# argtypes per exported function, in header order.
SIGNATURES: dict[str, tuple[object, list]] = {
    "hb_version": (c_int, []),
    "hb_last_error": (ctypes.c_char_p, []),
    "hb_device_status": (c_int, [ctypes.POINTER(c_uint32), c_int]),
    "hb_selftest_wait_timeout": (c_int, [I64, P, P]),
    "hb_tick_pack": (c_int, [P, I32, P, I32, P, I32, I32, I32, I32, I32, I32, I32, I32, I32, I32,
                             P, P, P, P, P, P, P, P, I32, P, I32, P, I32, P, I32, P, P, P]),
    "hb_qk_norm_rope_append": (c_int, [P, I64, I64, P, I64, I64, P, I64, I64, P, P, F32, P, P, I64, P, P,
                                       P, P, P, I64, I32, I32, I32, I32, P]),
    "hb_attention_workspace_bytes": (c_size_t, [I32, I32, I32]),
    "hb_paged_attention": (c_int, [P, P, P, I64, I32, P, I32, P, P, I32, P, P, I32, P, I32, P, I32, P, I32, I32,
                                   I32, I32, I32, I32, F32, P, c_size_t, P, P]),
    "hb_paged_attention_static_workspace": (c_int, [P, P, P, I64, I32, P, I32, P, P, I32, P, P, I32, P, I32, P, I32,
                                                    P, I32, I32, I32, I32, I32, I32, F32, P, P]),
    "hb_rmsnorm": (c_int, [P, I64, P, P, F32, P, I32, I32, P]),
    "hb_add_rmsnorm": (c_int, [P, P, P, F32, P, P, I32, I32, P]),
    "hb_swiglu": (c_int, [P, P, I64, I64, P]),
    "hb_gemm_swiglu": (c_int, [P, I32, I32, P, I32, P, P]),
    "hb_attention_set_overlap": (c_int, [I32]),
    "hb_hash_token_blocks": (c_int, [P, P, I32, I32, P, P, P]),
    "hb_prefix_index_insert": (c_int, [P, I32, P, P, I32, P]),
    "hb_prefix_index_remove": (c_int, [P, I32, P, I32, P]),
    "hb_prefix_index_lookup": (c_int, [P, I32, P, P, P, I32, P, P, P]),
    "hb_lm_head_argmax": (c_int, [P, I32, I32, P, I32, P, P, P]),
    "hb_embedding": (c_int, [P, P, I64, P, I64, I32, P]),
    "hb_page_copy": (c_int, [P, I64, I32, I64, I64, P, P, I32, P]),
    "hb_sample": (c_int, [P, I64, I32, I32, P, P, P, P, P]),
    "hb_verify_drafts": (c_int, [P, P, P, P, I32, P, P, P]),
}


class NativeLibraryError(RuntimeError):
    """The CUDA library is missing or unusable; there is no CPU fallback."""


_lib = None


def header_symbols() -> list[str]:
    """Names the public header declares with HB_API."""
    text = HEADER.read_text()
    return re.findall(r"^HB_API\s+[\w\s\*]+?\b(hb_\w+)\(", text, flags=re.M)


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise NativeLibraryError(
            f"{LIB_PATH.name} is not built; run `python -m helios_b200.build` (nvcc, sm_100a)")
    try:
        lib = ctypes.CDLL(str(LIB_PATH))
    except OSError as error:  # pragma: no cover - depends on the host
        raise NativeLibraryError(f"cannot load {LIB_PATH}: {error}") from error
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    if lib.hb_version() != 1:
        raise NativeLibraryError("libhelios_b200 version mismatch")
    _lib = lib
    return lib


def last_error() -> str:
    return load().hb_last_error().decode(errors="replace")


def check(rc: int, what: str) -> None:
    """Raise the reference's exception types for a non-zero status."""
    if rc == HB_OK:
        return
    message = f"{what}: {last_error()}"
    if rc in (HB_ERR_INVALID, HB_ERR_UNSUPPORTED):
        raise ValueError(message)
    raise RuntimeError(message)


def device_status(clear: bool = True) -> int:
    """Synchronise and return (optionally clearing) the kernels' device status bits."""
    value = c_uint32(0)
    check(load().hb_device_status(ctypes.byref(value), int(clear)), "hb_device_status")
    return int(value.value)


def describe_status(bits: int) -> list[str]:
    return [text for bit, text in STATUS_BITS.items() if bits & bit]
