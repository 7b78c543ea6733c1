"""ctypes binding of libh3sa.so, the C ABI declared in include/h3sa.h.

The library is the only compute path: importing this module without the built library
raises, and every wrapper raises RuntimeError with the library's message on a non-zero
status. Tensors cross the boundary as raw device pointers; the stream is torch's current
CUDA stream unless one is given.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

_LIB_PATH = Path(os.environ.get("H3SA_LIBRARY", Path(__file__).resolve().parent / "libh3sa.so"))

H3SA_OK = 0
H3SA_ERR_INVALID = 1
H3SA_ERR_UNSUPPORTED = 2
H3SA_ERR_CUDA = 3

DEVERR_WAIT_TIMEOUT = 1
DEVERR_BAD_PAGE = 2
DEVERR_BAD_INDEX = 4

MAX_PROBLEMS = 4


class Problem(ctypes.Structure):
    _fields_ = [
        ("q_lo", ctypes.c_int32),
        ("q_hi", ctypes.c_int32),
        ("kv_lo", ctypes.c_int32),
        ("kv_hi", ctypes.c_int32),
        ("sparse", ctypes.c_int32),
        ("reserved", ctypes.c_int32 * 3),
    ]


class MaskPolicy(ctypes.Structure):
    _fields_ = [
        ("mode", ctypes.c_int32),
        ("n_hist", ctypes.c_int32),
        ("n_kv", ctypes.c_int32),
        ("sinks", ctypes.c_int32),
        ("window", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("density", ctypes.c_double),
        ("q_block_audio", ctypes.c_void_p),
        ("kv_block_audio", ctypes.c_void_p),
    ]


class Rows(ctypes.Structure):
    _fields_ = [
        ("base", ctypes.c_void_p),
        ("paged", ctypes.c_int32),
        ("extent", ctypes.c_int32),
        ("page_table", ctypes.c_void_p),
        ("table_blocks", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


_P = ctypes.c_void_p
_I = ctypes.c_int32
_F = ctypes.c_float

# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "h3sa_abi_version": (ctypes.c_int, []),
    "h3sa_last_error": (ctypes.c_char_p, []),
    "h3sa_attention_smem_bytes": (ctypes.c_size_t, [ctypes.c_int]),
    "h3sa_attention_fwd": (
        ctypes.c_int,
        [_P, _P, _I, _I, _I, _P, _P, _I, _P, _I, ctypes.POINTER(Problem), _I, _F,
         _P, _P, _I, _I, _P, _P],
    ),
    "h3sa_attention_fwd_fp8": (
        ctypes.c_int,
        [_P, _P, _I, _I, _I, _P, _P, _I, _P, _I, ctypes.POINTER(Problem), _I, _F,
         _P, _P, _P, _P, _P, _I, _I, _P, _P],
    ),
    "h3sa_attention_fwd_fp8_parts": (
        ctypes.c_int,
        [_P, _P, _I, _I, _I, _P, _P, _I, _P, _I, ctypes.POINTER(Problem), _I, _F,
         _P, _P, _I, _P, _P, _P, _P, _I, _I, _P, _P],
    ),
    "h3sa_kv_copy_rows": (
        ctypes.c_int,
        [ctypes.POINTER(Rows), ctypes.POINTER(Rows), _I, _P, _I, _P, _I, _I, _I, _I, _P, _P],
    ),
    "h3sa_quantize_fp8_per_head": (ctypes.c_int, [_P, _P, _P, _I, _I, _I, _I, _P]),
    "h3sa_quantize_fp8_per_head_noalloc": (ctypes.c_int, [_P, _P, _P, _I, _I, _I, _I, _P]),
    "h3sa_quantize_fp8_rows": (
        ctypes.c_int,
        [ctypes.POINTER(Rows), ctypes.POINTER(Rows), _I, _I, _I, _I, _I, _P, _P, _P, _I, _P, _P]),
    "h3sa_quantize_fp8_pool": (ctypes.c_int, [_P, _P, _P, _I, _I, _P, _I, _I, _P, _P]),
    "h3sa_segment_row_means": (
        ctypes.c_int, [ctypes.POINTER(Rows), _P, _I, _I, _I, _P, _P, _P, _P]),
    "h3sa_commit_scores": (ctypes.c_int, [_P, _P, _I, _I, _P, _P]),
    "h3sa_sol_attention": (
        ctypes.c_int, [_P, _I, _P, _P, _I, _I, _I, _F, _F, _I, _P, _P, _P, _P, _P, _P, _P, _P]),
    "h3sa_w8a8_gemm": (ctypes.c_int, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _P]),
    "h3sa_quantize_int8_rows": (ctypes.c_int, [_P, _P, _P, _I, _I, _I, _P]),
    "h3sa_gemm_bf16": (ctypes.c_int, [_P, _P, _P, _I, _I, _I, _I, _P, _I, _I, _P, _P]),
    "h3sa_tp_reduce": (ctypes.c_int, [_P, _P, _I, _I, _I, _I, _P]),
    "h3sa_qkv_norm_rope": (ctypes.c_int, [_P, _P, _P, _P, _I, _I, _P, _I, _I, _I, _F, _P, _P]),
    "h3sa_qkv_norm_rope_pack": (
        ctypes.c_int, [_P, _P, _P, _P, _P, _I, _I, _P, _I, _I, _I, _I, _F, _P, _P]),
    "h3sa_qkv_norm_rope_scatter_paged": (
        ctypes.c_int, [_P, _P, _P, _P, _I, _I, _P, _I, _I, _I, _I, _I, _P, _P, _P, _I, _P, _I, _I,
                       _F, _P, _P]),
    "h3sa_qkv_norm_rope_amax": (
        ctypes.c_int, [_P, _P, _P, _P, _I, _I, _P, _I, _I, _I, _P, _P, _F, _P, _P]),
    "h3sa_qkv_norm_rope_scatter_fp8": (
        ctypes.c_int, [_P, _P, _P, _P, _I, _I, _P, _I, _I, _I, _I, _I, _P, _I, _P, _I, _P, _P, _P,
                       _I, _P, _I, _I, _P, _P, _P, _P, _P, _P, _I, _P, _I, _I, _F, _P, _P]),
    "h3sa_publish_words": (ctypes.c_int, [_P, _P, _I, _I, _I, _P]),
    "h3sa_block_mask": (
        ctypes.c_int,
        [_P, _I, _I, _I, _I, _I, _P, _I, _P, _I, ctypes.POINTER(MaskPolicy), _P, _P, _I, _P, _P],
    ),
    "h3sa_attention_fwd_scatter": (
        ctypes.c_int,
        [_P, _I, _I, _I, _P, _P, _I, _P, _I, ctypes.POINTER(Problem), _I, _F, _P, _P, _I, _I,
         _P, _I, _I, _I, _I, _P, _P],
    ),
    "h3sa_peer_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]),
    "h3sa_peer_free": (ctypes.c_int, [_P]),
    "h3sa_ipc_handle": (ctypes.c_int, [_P, _P]),
    "h3sa_ipc_open": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    "h3sa_ipc_close": (ctypes.c_int, [_P]),
    "h3sa_scatter_qkv": (ctypes.c_int, [_P, _I, _I, _I, _I, _I, _P, _P]),
    "h3sa_scatter_qkv_paged": (ctypes.c_int,
                               [_P, _I, _I, _I, _I, _I, _P, _P, _P, _I, _P, _I, _I, _P, _P]),
    "h3sa_peer_barrier": (ctypes.c_int, [_P, _I, _I, ctypes.c_uint32, _P, _P]),
    "h3sa_peer_barrier_limit": (ctypes.c_int, [_P, _I, _I, ctypes.c_uint32, ctypes.c_int64, _P,
                                               _P]),
    "h3sa_permute_rows": (
        ctypes.c_int,
        [_P, _P, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64),
         ctypes.POINTER(ctypes.c_int64), _I, _P],
    ),
}


def library_path() -> Path:
    return _LIB_PATH


def _load() -> ctypes.CDLL:
    if not _LIB_PATH.exists():
        raise ImportError(
            f"h3sa: native library {_LIB_PATH} is missing; build it with "
            "`python taomate-h3_b200/build.py` (there is no fallback path)"
        )
    lib = ctypes.CDLL(str(_LIB_PATH))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


LIB = _load()


def last_error() -> str:
    msg = LIB.h3sa_last_error()
    return msg.decode() if msg else ""


class H3SAError(RuntimeError):
    """A non-zero status from the C ABI."""

    def __init__(self, fn: str, code: int) -> None:
        super().__init__(f"{fn} failed with status {code}: {last_error()}")
        self.code = code


def check(fn: str, code: int) -> None:
    if code != H3SA_OK:
        raise H3SAError(fn, code)


def call(name: str, *args: object) -> None:
    check(name, getattr(LIB, name)(*args))


def stream_handle(stream: object | None = None) -> int:
    import torch

    s = torch.cuda.current_stream() if stream is None else stream
    return int(s.cuda_stream)


def ptr(t: object | None) -> int | None:
    if t is None:
        return None
    return int(t.data_ptr())  # type: ignore[attr-defined]
