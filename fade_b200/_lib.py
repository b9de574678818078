"""ctypes binding of libfade_sm100.so (the C ABI declared in include/fade_b200.h).

Every call passes raw device pointers, sizes, strides and the current torch
CUDA stream.  Status codes are mapped to the exception types and messages the
reference raises for the same conditions (``ValueError`` for bad shapes,
``RuntimeError`` otherwise).  There is no CPU fallback: a missing library or a
CPU tensor raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libfade_sm100.so"

FADE_OK = 0
FADE_ERR_INVALID_ARG = 1
FADE_ERR_ODD_DIM = 2
FADE_ERR_GROUP = 3
FADE_ERR_UNSUPPORTED = 4
FADE_ERR_ALIGN = 5
FADE_ERR_WORKSPACE = 6
FADE_ERR_CUDA = 7
FADE_ERR_TIMEOUT = 8

FADE_F16 = 0
FADE_BF16 = 1
FADE_F32 = 2

SEG_FP = 0
SEG_INT4 = 1
SEG_INT4K_INT2V = 2
SEG_ROT = 3
MAX_SEGMENTS = 4

_c_i64 = ctypes.c_int64
_vp = ctypes.c_void_p


class View4(ctypes.Structure):
    _fields_ = [(n, _c_i64) for n in ("B", "H", "S", "D", "sb", "sh", "ss", "sd")]


class KVSegment(ctypes.Structure):
    _fields_ = [
        ("kind", ctypes.c_int32),
        ("bits", ctypes.c_int32),
        ("group", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("k", _vp),
        ("v", _vp),
        ("k_scale", _vp),
        ("v_scale", _vp),
        ("row_sb", _c_i64),
        ("row_sh", _c_i64),
        ("row_base", _vp),
        ("lens", _vp),
        ("len", _c_i64),
        ("max_len", _c_i64),
        ("ks_sb", _c_i64),
        ("ks_sh", _c_i64),
        ("n_rows", _c_i64),
        ("page_table", _vp),
        ("pages_per_row", _c_i64),
    ]


PAGE_TOKENS = 128


class DecodeDesc(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int32),
        ("B", ctypes.c_int32),
        ("Hq", ctypes.c_int32),
        ("Hkv", ctypes.c_int32),
        ("D", ctypes.c_int32),
        ("n_q", ctypes.c_int32),
        ("sm_scale", ctypes.c_float),
        ("q", _vp),
        ("q_sb", _c_i64),
        ("q_sh", _c_i64),
        ("q_ss", _c_i64),
        ("out", _vp),
        ("o_sb", _c_i64),
        ("o_sh", _c_i64),
        ("o_ss", _c_i64),
        ("rotation", _vp),
        ("n_segments", ctypes.c_int32),
        ("n_ctas", ctypes.c_int32),
        ("cu_units", _vp),
        ("seg", KVSegment * MAX_SEGMENTS),
    ]


class AgeOutDesc(ctypes.Structure):
    _fields_ = [
        ("ring_seg", ctypes.c_int32),
        ("mid_seg", ctypes.c_int32),
        ("ring_cap", _c_i64),
        ("ring_origin", _c_i64),
        ("k_new", _vp),
        ("v_new", _vp),
        ("new_sb", _c_i64),
        ("new_sh", _c_i64),
        ("prefetch_tiers", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


# (name, restype, argtypes) for every symbol of include/fade_b200.h
_SIGNATURES = {
    "fade_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "fade_version": (ctypes.c_int, []),
    "fade_last_cuda_error": (ctypes.c_int, []),
    "fade_set_device": (ctypes.c_int, [ctypes.c_int]),
    "fade_sm_count": (ctypes.c_int, []),
    "fade_quant_int4_k": (ctypes.c_int, [_vp, ctypes.c_int, View4, _vp, _vp, _vp]),
    "fade_quant_int4_v": (ctypes.c_int, [_vp, ctypes.c_int, View4, _vp, _vp, _vp]),
    "fade_quant_int2_grouped": (
        ctypes.c_int,
        [_vp, ctypes.c_int, View4, ctypes.c_int, _vp, _vp, _vp, _vp],
    ),
    "fade_pack_codes": (ctypes.c_int, [_vp, _c_i64, _c_i64, ctypes.c_int, _vp, _vp]),
    "fade_unpack_codes": (ctypes.c_int, [_vp, _c_i64, _c_i64, ctypes.c_int, _vp, _vp]),
    "fade_dequant": (
        ctypes.c_int,
        [_vp, ctypes.c_int, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
         _c_i64, _c_i64, _c_i64, _c_i64, _vp, _vp],
    ),
    "fade_rotated_quant": (
        ctypes.c_int,
        [_vp, ctypes.c_int, View4, _vp, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp,
         ctypes.c_size_t, _vp],
    ),
    "fade_rotated_quant_check": (ctypes.c_int, [_vp]),
    "fade_rotated_dequant": (
        ctypes.c_int,
        [_vp, ctypes.c_int, _vp, ctypes.c_int, _vp, ctypes.c_int, _c_i64, _c_i64, _c_i64,
         _c_i64, _vp, _vp],
    ),
    "fade_rerope_gather": (
        ctypes.c_int,
        [_vp, _vp, ctypes.c_int, View4, _vp, _c_i64, _vp, _vp, _vp, _vp, ctypes.c_int, _vp,
         _vp, _vp],
    ),
    "fade_age_out_int4": (
        ctypes.c_int,
        [_vp, _vp, ctypes.c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
         _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _vp, _vp, _vp, _c_i64, _c_i64, _vp],
    ),
    "fade_decode_attn_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(DecodeDesc)]),
    "fade_decode_attn": (
        ctypes.c_int,
        [ctypes.POINTER(DecodeDesc), _vp, ctypes.c_size_t, _vp],
    ),
    "fade_decode_attn_age_out": (
        ctypes.c_int,
        [ctypes.POINTER(DecodeDesc), ctypes.POINTER(AgeOutDesc), _vp, ctypes.c_size_t, _vp],
    ),
    "fade_workspace_check": (ctypes.c_int, [_vp, ctypes.c_size_t, _vp]),
    "fade_decode_attn_noalloc_max_bytes": (ctypes.c_size_t, []),
    "fade_decode_attn_noalloc": (ctypes.c_int, [ctypes.POINTER(DecodeDesc), _vp]),
    "fade_decode_attn_noalloc_check": (ctypes.c_int, [_vp]),
    "fade_set_middle_kernel": (ctypes.c_int, [ctypes.c_int]),
    "fade_get_middle_kernel": (ctypes.c_int, []),
}

_lib = None
_lock = threading.Lock()


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """Load the shared library once.  Raises if it has not been built."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        if path is None and os.environ.get("FADE_LIB_PATH"):
            path = os.environ["FADE_LIB_PATH"]   # alternative build (profiling)
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"{p.name} is missing: build it with `python -m fade_b200.csrc.build` "
                "(fade_b200 has no CPU fallback)"
            )
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def symbols() -> list[str]:
    return list(_SIGNATURES)


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------
_DTYPE_CODE = {torch.float16: FADE_F16, torch.bfloat16: FADE_BF16, torch.float32: FADE_F32}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dt]
    except KeyError as e:
        raise ValueError(f"unsupported dtype {dt}; expected float16, bfloat16 or float32") from e


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                "fade_b200 kernels run on CUDA tensors only (sm_100a); got a tensor on "
                f"{t.device}. There is no CPU path."
            )
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} vs {t.device}")
    if dev is None:
        raise RuntimeError("no CUDA tensor given")
    return dev


_tls = threading.local()


def bind(device: torch.device) -> int:
    """Make `device` current for the library; returns the current stream handle."""
    lib = load()
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if getattr(_tls, "dev", None) != idx:
        check(lib.fade_set_device(idx), "fade_set_device")
        _tls.dev = idx
    return torch.cuda.current_stream(idx).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def view4(t: torch.Tensor) -> View4:
    if t.dim() != 4:
        raise ValueError(f"expected a 4-D [B, H, S, D] tensor, got shape {tuple(t.shape)}")
    B, H, S, D = t.shape
    sb, sh, ss, sd = t.stride()
    return View4(B, H, S, D, sb, sh, ss, sd)


class FadeKernelError(RuntimeError):
    pass


def check(status: int, what: str, value_error_msg: str | None = None) -> None:
    if status == FADE_OK:
        return
    lib = load()
    msg = lib.fade_status_string(status).decode()
    if status in (FADE_ERR_ODD_DIM, FADE_ERR_GROUP, FADE_ERR_INVALID_ARG):
        raise ValueError(value_error_msg or f"{what}: {msg}")
    if status == FADE_ERR_CUDA:
        msg += f" (cudaError {lib.fade_last_cuda_error()})"
    raise FadeKernelError(f"{what}: {msg}")
