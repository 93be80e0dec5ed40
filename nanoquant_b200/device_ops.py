"""Device-side layout-v1 helpers backed by ``libnqb.so``.

``pack_signs_cuda`` / ``unpack_signs_cuda`` run layout-v1 packing on the GPU
(the reference does it on the CPU: ``src/nanoquant/runtime/packed.py:170-218``);
``decode_product_codebook_cuda`` expands a product-codebook right factor on the
GPU (reference ``product_codebook.py:110-143``).  They exist so the bit-level
work of the CUDA path can be checked bit-exactly against the host format code.
"""

from __future__ import annotations

import ctypes

import torch

from nanoquant_b200 import _native
from nanoquant_b200.packed import packed_word_count


def _require_cuda(value: torch.Tensor, name: str) -> None:
    if value.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor")
    if not value.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def pack_signs_cuda(signs: torch.Tensor) -> torch.Tensor:
    """+/-1 matrix on the GPU -> layout-v1 int32 words on the GPU."""

    _require_cuda(signs, "signs")
    if signs.ndim != 2:
        raise ValueError("signs must be a matrix")
    rows, cols = signs.shape
    words = torch.empty((rows, packed_word_count(cols)), dtype=torch.int32, device=signs.device)
    _native.call(
        "nqb_pack_signs",
        signs.data_ptr(),
        _native.dtype_code(signs.dtype),
        rows,
        cols,
        words.data_ptr(),
        _native.current_stream_handle(signs.device),
    )
    return words


def unpack_signs_cuda(words: torch.Tensor, rows: int, columns: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Layout-v1 words on the GPU -> (fp32 +/-1 matrix, count of rows with non-zero padding)."""

    _require_cuda(words, "words")
    if words.dtype != torch.int32 or tuple(words.shape) != (rows, packed_word_count(columns)):
        raise ValueError("words must be int32 [rows, ceil(columns/32)]")
    signs = torch.empty((rows, columns), dtype=torch.float32, device=words.device)
    bad = torch.zeros((1,), dtype=torch.int32, device=words.device)
    _native.call(
        "nqb_unpack_signs",
        words.data_ptr(),
        rows,
        columns,
        signs.data_ptr(),
        bad.data_ptr(),
        _native.current_stream_handle(words.device),
    )
    return signs, bad


def decode_product_codebook_cuda(
    free_words: torch.Tensor,
    payload: torch.Tensor,
    first: torch.Tensor,
    second: torch.Tensor,
    *,
    rank: int,
    columns: int,
) -> torch.Tensor:
    """Product-codebook right factor on the GPU -> layout-v1 words [rank, ceil(columns/32)]."""

    for name, value in (("free_words", free_words), ("payload", payload), ("first", first), ("second", second)):
        _require_cuda(value, name)
    out = torch.empty((rank, packed_word_count(columns)), dtype=torch.int32, device=free_words.device)
    _native.call(
        "nqb_decode_product_codebook",
        free_words.data_ptr(),
        free_words.shape[0],
        rank,
        columns,
        payload.data_ptr(),
        first.data_ptr(),
        second.data_ptr(),
        out.data_ptr(),
        _native.current_stream_handle(free_words.device),
    )
    return out


def decode_mixed_v_cuda(
    free_words: torch.Tensor,
    payload: torch.Tensor,
    codebook: torch.Tensor,
    *,
    rank: int,
    columns: int,
) -> torch.Tensor:
    """Mixed-V right factor on the GPU -> layout-v1 words [rank, ceil(columns/32)] (``nqb_decode_mixed_v``).

    The records must be valid (``MixedVLayerState`` validates them on
    construction); the kernel stays in bounds for any payload.
    """

    for name, value in (("free_words", free_words), ("payload", payload), ("codebook", codebook)):
        _require_cuda(value, name)
        if value.dtype != torch.int32 or not value.is_contiguous():
            raise ValueError(f"mixed-V {name} must be contiguous int32")
    words_per_row = packed_word_count(columns)
    free_rows = int(free_words.shape[0])
    if tuple(free_words.shape) != (free_rows, words_per_row) or tuple(codebook.shape) != (1024,):
        raise ValueError("mixed-V free words or codebook shape differs")
    if payload.numel() * 32 < (rank - free_rows) * words_per_row * 19:
        raise ValueError("mixed-V payload is shorter than its records")
    out = torch.empty((rank, words_per_row), dtype=torch.int32, device=free_words.device)
    _native.call(
        "nqb_decode_mixed_v",
        free_words.data_ptr(),
        free_rows,
        rank,
        columns,
        payload.data_ptr(),
        codebook.data_ptr(),
        out.data_ptr(),
        _native.current_stream_handle(free_words.device),
    )
    return out


def repack_mixed_v_cuda(payload: torch.Tensor, *, rank: int, columns: int, free_rows: int) -> torch.Tensor:
    """Coded mixed-V tiles for decode programs (``nqb_repack_mixed_v``) -> uint8 bytes.

    Tiles of 128 rows from ``ceil(free_rows / 128)`` on keep their records,
    widened to 20 bits with the pair id resolved (index | a << 10 | b << 15):
    per 256-column slice, row ``r``'s 8 records back to back from bit ``160 r``
    (2560 bytes per tile slice).
    """

    _require_cuda(payload, "payload")
    if payload.dtype != torch.int32 or not payload.is_contiguous():
        raise ValueError("mixed-V payload must be contiguous int32")
    if payload.numel() * 32 < (rank - free_rows) * packed_word_count(columns) * 19:
        raise ValueError("mixed-V payload is shorter than its records")
    size = ctypes.c_size_t(0)
    _native.call("nqb_mixed_v_tiles_bytes", rank, columns, free_rows, ctypes.byref(size))
    out = torch.zeros(max(size.value, 16), dtype=torch.uint8, device=payload.device)
    if size.value:
        _native.call("nqb_repack_mixed_v", payload.data_ptr(), rank, columns, free_rows, out.data_ptr(),
                     _native.current_stream_handle(payload.device))
    return out


def repack_product_codebook_cuda(payload: torch.Tensor, first: torch.Tensor, second: torch.Tensor, *, rank: int,
                                 columns: int, free_rows: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Coded product-codebook tiles and their decode table (``nqb_repack_product_codebook``).

    Returns ``(tiles, table)``: tiles of 128 rows from ``ceil(free_rows /
    128)`` on keep one 16-bit record per word, per 256-column slice row ``r``'s
    8 records at byte ``16 r`` (2048 bytes per tile slice); ``table`` is int32
    ``[1024]``: the first half words, the second half words shifted to bits
    16..31, zeros.
    """

    for name, value in (("payload", payload), ("first", first), ("second", second)):
        _require_cuda(value, name)
    if payload.dtype != torch.int32 or not payload.is_contiguous():
        raise ValueError("product-codebook payload must be contiguous int32")
    for name, value in (("first", first), ("second", second)):
        if value.dtype != torch.int16 or value.shape != (256,) or not value.is_contiguous():
            raise ValueError(f"product-codebook {name} half table must be contiguous int16 [256]")
    if payload.numel() * 2 < (rank - free_rows) * packed_word_count(columns):
        raise ValueError("product-codebook payload is shorter than its records")
    size = ctypes.c_size_t(0)
    _native.call("nqb_product_codebook_tiles_bytes", rank, columns, free_rows, ctypes.byref(size))
    tiles = torch.zeros(max(size.value, 16), dtype=torch.uint8, device=payload.device)
    table = torch.empty(1024, dtype=torch.int32, device=payload.device)
    _native.call("nqb_repack_product_codebook", payload.data_ptr(), first.data_ptr(), second.data_ptr(), rank,
                 columns, free_rows, tiles.data_ptr(), table.data_ptr(), _native.current_stream_handle(payload.device))
    return tiles, table
