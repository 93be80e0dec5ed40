"""ctypes binding of ``libnqb.so`` (declarations in ``include/nqb.h``).

The library is loaded from the package's ``_lib`` directory and nowhere else;
if it is missing, :func:`library` raises, so no caller can silently fall back
to another implementation.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

from nanoquant_b200.build import LIB_PATH, TRACE_LIB_PATH

NQB_OK = 0
NQB_ERR_INVALID_ARGUMENT = 1
NQB_ERR_ALIGNMENT = 2
NQB_ERR_DTYPE = 3
NQB_ERR_CUDA = 4
NQB_ERR_WORKSPACE = 5
NQB_ERR_UNSUPPORTED = 6
NQB_ERR_TIMEOUT = 7

NQB_PATH_GENERIC = 0
NQB_PATH_TENSOR_CORE = 1
NQB_PATH_PREFILL = 2

NQB_F32 = 0
NQB_F16 = 1
NQB_BF16 = 2
NQB_I8 = 3
NQB_I32 = 4
NQB_X_SWIGLU = 16  # program-op input: silu(x) * x2, both fp32
NQB_X_GEGLU = 17  # program-op input: gelu_tanh(x) * x2, both fp32
NQB_CODED_MIXED_V = 0  # nqb_linear_desc.coded_format
NQB_CODED_PRODUCT_CODEBOOK = 1
ABI_VERSION = 5  # the NQB_ABI_VERSION whose structs this module lays out

DTYPE_CODES = {
    torch.float32: NQB_F32,
    torch.float16: NQB_F16,
    torch.bfloat16: NQB_BF16,
    torch.int8: NQB_I8,
    torch.int32: NQB_I32,
}

_c_void_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32


class LinearDesc(ctypes.Structure):
    """Mirror of ``nqb_linear_desc`` (field order and types must match nqb.h)."""

    _fields_ = [
        ("in_features", _i64),
        ("out_features", _i64),
        ("rank", _i64),
        ("left_words", _c_void_p),
        ("right_words", _c_void_p),
        ("scale_pre", _c_void_p),
        ("scale_mid", _c_void_p),
        ("scale_post", _c_void_p),
        ("scale_dtype", _i32),
        ("bias", _c_void_p),
        ("bias_dtype", _i32),
        ("outlier_count", _i64),
        ("outlier_indices", _c_void_p),
        ("outlier_values", _c_void_p),
        ("outlier_value_dtype", _i32),
        ("outlier_scales", _c_void_p),
        ("overlay_rows", _i64),
        ("overlay_row_ids", _c_void_p),
        ("overlay_values", _c_void_p),
        ("overlay_scales", _c_void_p),
        ("overlay_scale_dtype", _i32),
        ("codebook_free_rows", _i64),
        ("codebook_free_words", _c_void_p),
        ("codebook_payload", _c_void_p),
        ("codebook_first", _c_void_p),
        ("codebook_second", _c_void_p),
        ("left_tiles", _c_void_p),
        ("right_tiles", _c_void_p),
        ("patch_rank", ctypes.c_int64),
        ("patch_left", _c_void_p),
        ("patch_right", _c_void_p),
        ("patch_dtype", ctypes.c_int32),
        ("coded_right_tiles", _c_void_p),
        ("coded_codebook", _c_void_p),
        ("coded_free_rows", ctypes.c_int64),
        ("coded_format", ctypes.c_int32),
    ]


NQB_OP_LINEAR = 0
NQB_OP_ATTENTION = 1
NQB_EPI_STORE = 0
NQB_EPI_RESIDUAL = 1
NQB_EPI_QK_ROPE = 2


class ProgramOpExt(ctypes.Structure):
    """Mirror of ``nqb_program_op_ext``."""

    _fields_ = [
        ("kind", _i32),
        ("epilogue", _i32),
        ("norm_stats", _c_void_p),
        ("norm_weight", _c_void_p),
        ("norm_weight_dtype", _i32),
        ("eps", ctypes.c_float),
        ("out_stats", _c_void_p),
        ("q_heads", _i32),
        ("kv_heads", _i32),
        ("head_dim", _i32),
        ("q_norm_weight", _c_void_p),
        ("k_norm_weight", _c_void_p),
        ("qk_norm_dtype", _i32),
        ("cos_table", _c_void_p),
        ("sin_table", _c_void_p),
        ("q", _c_void_p),
        ("k_cache", _c_void_p),
        ("v_cache", _c_void_p),
        ("cache_len", _i64),
        ("position", _i64),
        ("attn_out", _c_void_p),
        ("sequence_stride", _i64),
    ]


class ProgramOp(ctypes.Structure):
    """Mirror of ``nqb_program_op``."""

    _fields_ = [
        ("layers", ctypes.POINTER(LinearDesc)),
        ("count", _i32),
        ("x", _c_void_p),
        ("x_dtype", _i32),
        ("y", ctypes.POINTER(_c_void_p)),
        ("x2", _c_void_p),
        ("ext", ctypes.POINTER(ProgramOpExt)),
    ]


# name -> (restype, argtypes); every symbol declared in include/nqb.h


SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "nqb_abi_version": (ctypes.c_int, []),
    "nqb_last_error": (ctypes.c_char_p, []),
    "nqb_linear_workspace_bytes": (ctypes.c_int, [ctypes.POINTER(LinearDesc), _i64, ctypes.POINTER(ctypes.c_size_t)]),
    "nqb_linear": (
        ctypes.c_int,
        [ctypes.POINTER(LinearDesc), _c_void_p, _i32, _i64, _c_void_p, _c_void_p, ctypes.c_size_t, _c_void_p],
    ),
    "nqb_linear_noalloc": (
        ctypes.c_int,
        [ctypes.POINTER(LinearDesc), _c_void_p, _i32, _i64, _c_void_p, _c_void_p],
    ),
    "nqb_grouped_workspace_bytes": (
        ctypes.c_int,
        [ctypes.POINTER(LinearDesc), _i32, _i64, ctypes.POINTER(ctypes.c_size_t)],
    ),
    "nqb_grouped_linear": (
        ctypes.c_int,
        [
            ctypes.POINTER(LinearDesc),
            _i32,
            _c_void_p,
            _i32,
            _i64,
            ctypes.POINTER(_c_void_p),
            _c_void_p,
            ctypes.c_size_t,
            _c_void_p,
        ],
    ),
    "nqb_patch_accumulate": (
        ctypes.c_int,
        [_c_void_p, _i32, _i64, _i64, _i64, _i64, _c_void_p, _c_void_p, _i32, _c_void_p, _c_void_p,
         ctypes.c_size_t, _c_void_p],
    ),
    "nqb_pack_signs": (ctypes.c_int, [_c_void_p, _i32, _i64, _i64, _c_void_p, _c_void_p]),
    "nqb_unpack_signs": (ctypes.c_int, [_c_void_p, _i64, _i64, _c_void_p, _c_void_p, _c_void_p]),
    "nqb_repack_bytes": (ctypes.c_int, [_i64, _i64, ctypes.POINTER(ctypes.c_size_t)]),
    "nqb_repack_signs": (ctypes.c_int, [_c_void_p, _i64, _i64, _c_void_p, _c_void_p]),
    "nqb_device_status": (ctypes.c_int, [ctypes.POINTER(_i32)]),
    "nqb_program_create": (ctypes.c_int, [ctypes.POINTER(ProgramOp), _i32, _i64, ctypes.POINTER(_c_void_p)]),
    "nqb_program_workspace_bytes": (ctypes.c_int, [_c_void_p, ctypes.POINTER(ctypes.c_size_t)]),
    "nqb_program_run": (ctypes.c_int, [_c_void_p, _c_void_p, ctypes.c_size_t, _c_void_p]),
    "nqb_program_run_dependent": (ctypes.c_int, [_c_void_p, _c_void_p, ctypes.c_size_t, _c_void_p]),
    "nqb_program_destroy": (ctypes.c_int, [_c_void_p]),
    "nqb_program_shape": (ctypes.c_int, [_c_void_p, ctypes.POINTER(_i32), ctypes.POINTER(_i32)]),
    "nqb_program_trace": (ctypes.c_int, [_c_void_p, ctypes.POINTER(_i64), ctypes.c_size_t]),
    "nqb_linear_path": (ctypes.c_int, [ctypes.POINTER(LinearDesc), _i32, _i32, _i64, ctypes.POINTER(_i32)]),
    "nqb_decode_product_codebook": (
        ctypes.c_int,
        [_c_void_p, _i64, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p],
    ),
    "nqb_decode_mixed_v": (ctypes.c_int, [_c_void_p, _i64, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p]),
    "nqb_mixed_v_tiles_bytes": (ctypes.c_int, [_i64, _i64, _i64, ctypes.POINTER(ctypes.c_size_t)]),
    "nqb_repack_mixed_v": (ctypes.c_int, [_c_void_p, _i64, _i64, _i64, _c_void_p, _c_void_p]),
    "nqb_product_codebook_tiles_bytes": (ctypes.c_int, [_i64, _i64, _i64, ctypes.POINTER(ctypes.c_size_t)]),
    "nqb_repack_product_codebook": (ctypes.c_int, [_c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _c_void_p,
                                                   _c_void_p, _c_void_p]),
    "nqb_rmsnorm": (ctypes.c_int, [_c_void_p, _c_void_p, _c_void_p, _i32, _i64, _i64, ctypes.c_float, _c_void_p, _i32,
                                   _c_void_p]),
    "nqb_qk_norm_rope": (ctypes.c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _c_void_p, _c_void_p,
                                        _i64, _i32, _i32, _i32, ctypes.c_float, _c_void_p, _c_void_p, _c_void_p, _i64,
                                        _i64, _c_void_p]),
    "nqb_decode_attention_workspace_bytes": (ctypes.c_int, [_i64, _i64, _i32, _i32, ctypes.POINTER(ctypes.c_size_t)]),
    "nqb_decode_attention": (ctypes.c_int, [_c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _i32, _i32, _i32,
                                            _c_void_p, _c_void_p, ctypes.c_size_t, _c_void_p]),
    "nqb_silu_mul": (ctypes.c_int, [_c_void_p, _c_void_p, _i64, _c_void_p, _i32, _c_void_p]),
    "nqb_gemv_bf16": (ctypes.c_int, [_c_void_p, _i64, _i64, _c_void_p, _i64, _c_void_p, _c_void_p]),
    "nqb_workspace_reset": (ctypes.c_int, [_c_void_p, ctypes.c_size_t, _c_void_p]),
    "nqb_residual_stats": (ctypes.c_int, [_c_void_p, _i64, _i64, _c_void_p, _c_void_p]),
    "nqb_rmsnorm_residual": (ctypes.c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i64, _i64,
                                            ctypes.c_float, _c_void_p, _i32, _c_void_p]),
    "nqb_decode_attention_window": (ctypes.c_int, [_c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _i32, _i32,
                                                   _i32, _i64, _c_void_p, _c_void_p, ctypes.c_size_t, _c_void_p]),
    "nqb_embedding_bf16": (ctypes.c_int, [_c_void_p, _i64, _c_void_p, _i64, _i64, ctypes.c_float, _c_void_p,
                                          _c_void_p]),
    "nqb_debug_set_barrier_limit": (ctypes.c_int, [ctypes.c_uint32]),
    "nqb_program_debug_barrier_skew": (ctypes.c_int, [_c_void_p, ctypes.c_uint32]),
}

_lock = threading.Lock()
_library: ctypes.CDLL | None = None


class NativeError(RuntimeError):
    """A libnqb call returned a non-zero status."""

    def __init__(self, function: str, status: int, message: str) -> None:
        super().__init__(f"{function} failed with status {status}: {message}")
        self.function = function
        self.status = status
        self.message = message


def library_path() -> Path:
    """The in-tree library; ``NQB_LIBRARY=trace`` selects the phase-trace build."""

    return TRACE_LIB_PATH if os.environ.get("NQB_LIBRARY") == "trace" else LIB_PATH


def library() -> ctypes.CDLL:
    """Load ``libnqb.so`` once; raises if the in-tree build is missing."""

    global _library
    with _lock:
        if _library is None:
            path = library_path()
            if not path.exists():
                raise RuntimeError(
                    f"{path.name} is not built at {path}; run `python -m nanoquant_b200.build`"
                )
            lib = ctypes.CDLL(str(path))
            for name, (restype, argtypes) in SIGNATURES.items():
                function = getattr(lib, name)
                function.restype = restype
                function.argtypes = argtypes
            if lib.nqb_abi_version() != ABI_VERSION:
                raise RuntimeError(f"{path.name} has ABI {lib.nqb_abi_version()}, this package lays out ABI "
                                   f"{ABI_VERSION}; rebuild with `python -m nanoquant_b200.build`")
            _library = lib
        return _library


def check(function: str, status: int) -> None:
    if status != NQB_OK:
        message = library().nqb_last_error().decode("utf-8", "replace")
        raise NativeError(function, status, message)


def call(function: str, *args: object) -> None:
    check(function, getattr(library(), function)(*args))


def current_stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(value: torch.Tensor | None) -> int | None:
    return None if value is None else value.data_ptr()


def dtype_code(dtype: torch.dtype) -> int:
    if dtype not in DTYPE_CODES:
        raise ValueError(f"dtype {dtype} has no libnqb code")
    return DTYPE_CODES[dtype]
