"""ctypes binding of libgdn_b200.so (the C ABI declared in include/gdn_b200.h).

There is no fallback: if the library is missing or does not export an entry
point, importing this module raises.  Build it with __graft_entry__.build()
(or `python track-c-gdn_b200/build.py`).
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

# GDN_B200_LIBRARY selects another build of the same library (the debug
# build with device-side index checks, libgdn_b200_debug.so).
LIB_PATH = Path(os.environ.get("GDN_B200_LIBRARY") or
                Path(__file__).resolve().parent / "libgdn_b200.so")

# Every symbol the header declares, with (restype, argtypes).
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_F = ctypes.c_float
SIGNATURES = {
    "gdn_b200_abi_version": (ctypes.c_int, []),
    "gdn_b200_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "gdn_b200_read_device_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int), _P]),
    "gdn_decode_qk4_v8_d128_k_last": (
        ctypes.c_int, [_P, _P, _P, _P, _P, _P, _P, _P, _F, _I64, _P, _P, _P]),
    "gdn_decode_mtp_qk4_v8_d128_k_last": (
        ctypes.c_int, [_P, _P, _P, _P, _P, _P, _P, _P, _F, _I64, _I64, _P, _P, _P, _P]),
    "gdn_decode_pool_qk4_v8_d128_k_last": (
        ctypes.c_int, [_P, _P, _P, _P, _I64, _P, _P, _P, _P, _P, _F, _I64, _I64, _P, _P]),
    "gdn_prefill_pool_qk4_v8_d128_k_last": (
        ctypes.c_int,
        [_P, _P, _P, _P, _I64, _P, _P, _P, _P, _P, _P, _I64, _I64, _F, _P, _P, ctypes.c_size_t, _P]),
    "gdn_decode_bf16_state_qk4_v8_d128_k_last": (
        ctypes.c_int, [_P, _P, _P, _P, _I64, _P, _P, _P, _P, _P, _F, _I64, _I64, _P, _P]),
    "gdn_prefill_workspace_bytes": (ctypes.c_size_t, [_I64, _I64]),
    "gdn_prefill_kernel_launches": (ctypes.c_int, [_I64, _I64]),
    "gdn_prefill_qk4_v8_d128_k_last": (
        ctypes.c_int,
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _F, _P, _P, _P, ctypes.c_size_t, _P]),
    "gdn_prefill_qk4_v8_d128_k_last_events": (
        ctypes.c_int,
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _F, _P, _P, _P, ctypes.c_size_t, _P,
         ctypes.c_int, _P]),
    "gdn_prefill_backward_workspace_bytes": (ctypes.c_size_t, [_I64, _I64]),
    "gdn_prefill_backward_kernel_launches": (ctypes.c_int, []),
    "gdn_prefill_backward_qk4_v8_d128_k_last": (
        ctypes.c_int,
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _F, _P, _P,
         _P, _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P]),
    "gdn_prefill_qk4_v8_d128_k_last_noalloc": (
        ctypes.c_int, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _F, _P, _P, _P]),
}

ABI_VERSION = 1

# Kernels each entry point launches per call (for launch accounting).
DECODE_KERNELS_PER_CALL = 1


class GdnError(RuntimeError):
    pass


def _load():
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is not built; run __graft_entry__.build() "
            "(the GDN kernels have no CPU or Triton fallback)")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)  # AttributeError if the export is missing
        fn.restype = res
        fn.argtypes = args
    if lib.gdn_b200_abi_version() != ABI_VERSION:
        raise ImportError(f"{LIB_PATH}: ABI version {lib.gdn_b200_abi_version()} != {ABI_VERSION}")
    return lib


lib = _load()


def check(status: int, what: str) -> None:
    if status != 0:
        msg = lib.gdn_b200_status_string(status).decode()
        raise GdnError(f"{what} failed: status {status} ({msg})")


def prefill_kernel_launches(total_tokens: int, num_seqs: int) -> int:
    """Kernels one prefill call launches for this problem size (3, or 5 when
    it runs the segmented evaluation)."""
    return int(lib.gdn_prefill_kernel_launches(int(total_tokens), int(num_seqs)))


def read_device_status(stream: int = 0) -> int:
    """Copy and clear the device status word (synchronises `stream`)."""
    code = ctypes.c_int(0)
    check(lib.gdn_b200_read_device_status(ctypes.byref(code), ctypes.c_void_p(stream)),
          "gdn_b200_read_device_status")
    return code.value
