"""ctypes binding of libwhistle_b200.so (include/whistle_b200.h).

The library is the product: every product below runs on the GPU through it.
There is no CPU fallback; a missing library or GPU raises.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libwhistle_b200.so"
HEADER = HERE.parent / "include" / "whistle_b200.h"

WC_OK, WC_ERR_INVALID, WC_ERR_UNSUPPORTED, WC_ERR_CUDA, WC_ERR_NOMEM, WC_ERR_DEVICE = range(6)


class WhistleError(Exception):
    """A failed call; .status is the wc_status code."""

    def __init__(self, status: int, msg: str):
        super().__init__(msg)
        self.status = status


class CQError(WhistleError, ValueError):
    """What the reference returns as an error (e.g. cq.New's validation)."""


class Panic(WhistleError, RuntimeError):
    """What the reference panics on (shape and range misuse)."""


class CudaError(WhistleError, RuntimeError):
    """A CUDA runtime failure, or a handle used on the wrong device."""


_c_void_p = ctypes.c_void_p
_c_int = ctypes.c_int
_c_size = ctypes.c_size_t
_c_float = ctypes.c_float

_SIGS = {
    "wc_last_error": (_c_size, [ctypes.c_char_p, _c_size]),
    "wc_version": (ctypes.c_char_p, []),
    "wc_launch_count": (ctypes.c_uint64, []),
    "wc_cq_create": (_c_int, [_c_void_p, _c_size, _c_void_p, _c_size, _c_void_p, _c_size, _c_int, _c_int, _c_int,
                              _c_int, _c_int, ctypes.POINTER(_c_void_p)]),
    "wc_cq_rows": (_c_int, [_c_void_p, _c_int, _c_int, ctypes.POINTER(_c_void_p)]),
    "wc_cq_exact": (_c_int, [_c_void_p, ctypes.POINTER(_c_void_p)]),
    "wc_cq_destroy": (None, [_c_void_p]),
    "wc_cq_out": (_c_int, [_c_void_p]),
    "wc_cq_in": (_c_int, [_c_void_p]),
    "wc_cq_bits": (_c_int, [_c_void_p]),
    "wc_cq_bytes": (_c_size, [_c_void_p]),
    "wc_cq_gemm": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_int, _c_void_p]),
    "wc_cq_gemm_host": (_c_int, [_c_void_p, _c_void_p, _c_size, _c_void_p, _c_size, _c_int]),
    "wc_cq_gemm_ex": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_int, _c_int, _c_void_p]),
    "wc_cq_gemms_ex": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_void_p, _c_int, _c_int, _c_void_p]),
    "wc_cq_prepare_tc": (_c_int, [_c_void_p]),
    "wc_cq_gemm_tc_noalloc": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_int, _c_void_p, _c_void_p]),
    "wc_device_status": (_c_int, [ctypes.POINTER(_c_int)]),
    "wc_testing_gemm_tc_stall": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_int, _c_void_p]),
    "wc_cq_gemms": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_void_p, _c_int, _c_void_p]),
    "wc_cq_gemms_host": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_size, _c_void_p, _c_void_p, _c_int]),
    "wc_cq_row": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_void_p]),
    "wc_cq_row_gather": (_c_int, [_c_void_p, _c_void_p, _c_int, _c_void_p, _c_void_p, _c_void_p]),
    "wc_cq_row_host": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_size]),
    "wc_quantize_rows": (_c_int, [_c_void_p, _c_int, _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p]),
    "wc_quantize_rows_host": (_c_int, [_c_void_p, _c_size, _c_int, _c_int, _c_void_p, _c_void_p]),
    "wc_head_argmax": (_c_int, [_c_void_p, _c_int, _c_int, _c_float, _c_void_p, _c_void_p, _c_void_p]),
    "wc_attend_int8": (_c_int, [_c_void_p, _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int, _c_int,
                                _c_int, _c_int, _c_void_p, _c_float, _c_int, _c_void_p, _c_void_p, _c_void_p]),
    "wc_attend_int8_host": (_c_int, [_c_void_p, _c_size, _c_int, _c_int, _c_void_p, _c_size, _c_void_p, _c_size,
                                     _c_void_p, _c_size, _c_void_p, _c_size, _c_int, _c_int, _c_int, _c_void_p,
                                     _c_float, _c_int, _c_void_p, _c_size, _c_void_p, _c_size]),
    "wc_attend_int8_streams": (_c_int, [_c_int, _c_void_p, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                        _c_int, _c_void_p, _c_int, _c_int, _c_int, _c_float, _c_int, _c_void_p,
                                        _c_void_p]),
    "wc_decoder_create": (_c_int, [_c_void_p, _c_int, _c_int, _c_int, _c_int, ctypes.POINTER(_c_void_p)]),
    "wc_decoder_destroy": (None, [_c_void_p]),
    "wc_decoder_memory": (_c_int, [_c_void_p, _c_void_p, _c_int, _c_int, _c_void_p]),
    "wc_decoder_extend": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p]),
    "wc_decoder_greedy": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_int, _c_int, _c_int, _c_void_p, _c_void_p,
                                   _c_void_p, _c_void_p, _c_void_p]),
    "wc_decoder_len": (_c_int, [_c_void_p]),
    "wc_decoder_memory_of": (_c_int, [_c_void_p, _c_int, ctypes.POINTER(_c_void_p), ctypes.POINTER(_c_void_p),
                                      ctypes.POINTER(_c_void_p), ctypes.POINTER(_c_void_p)]),
    "wc_decoder_memory_beams": (_c_int, [_c_void_p, _c_void_p, _c_int, _c_int, _c_int, _c_void_p]),
    "wc_beam_default": (None, [_c_void_p]),
    "wc_decoder_beam": (_c_int, [_c_void_p, _c_void_p, _c_int, _c_void_p, _c_int, _c_int, _c_void_p, _c_void_p,
                                 _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p]),
    "wc_encoder_create": (_c_int, [_c_void_p, _c_int, _c_int, _c_int, ctypes.POINTER(_c_void_p)]),
    "wc_encoder_destroy": (None, [_c_void_p]),
    "wc_encoder_stack": (_c_int, [_c_void_p, _c_void_p, _c_int, _c_int, _c_void_p, _c_void_p]),
    "wc_encoder_logmel": (_c_int, [_c_void_p, _c_void_p, _c_int, _c_int, _c_void_p, _c_void_p]),
    "wc_encoder_stem_frames": (_c_int, [_c_int]),
    "wc_encoder_stem": (_c_int, [_c_void_p, _c_void_p, _c_int, _c_int, _c_void_p, _c_void_p]),
    "wc_encoder_embed": (_c_int, [_c_void_p, _c_void_p, _c_int, _c_int, _c_void_p, _c_void_p]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library with its signatures set. Raises if it is missing."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python go-whistle_b200/build.py`")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().wc_last_error(buf, len(buf))
    return buf.value.decode()


def check(status: int) -> None:
    """Raises the error a non-zero wc_status stands for."""
    if status == WC_OK:
        return
    msg = last_error()
    if status == WC_ERR_INVALID:
        raise Panic(status, msg)
    if status == WC_ERR_UNSUPPORTED:
        raise CQError(status, msg)
    raise CudaError(status, msg)


def exported_symbols() -> list[str]:
    """The entry points the headers under include/ declare (the boundary,
    whistle_b200.h, and the test-only whistle_b200_testing.h)."""
    import re

    text = "\n".join(h.read_text() for h in sorted(HEADER.parent.glob("*.h")))
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(wc_\w+)\s*\(", text, re.M)))
