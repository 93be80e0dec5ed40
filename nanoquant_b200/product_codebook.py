"""Product-codebook right factor (``product-codebook-free-k16-v1``).

Restates ``src/nanoquant/runtime/product_codebook.py:1-307`` of the reference.
A layer keeps its first ``free_rows`` rows of ``V`` as plain layout-v1 words.
Every other word of ``V`` is a 16-bit record: the low byte indexes a 256-entry
table of 16-bit sign half-words for bits 0..15 of the word, the high byte a
second table for bits 16..31.  Records are packed two per int32 word, low half
first.  When the factorisation was fitted transposed, decoding transposes back to
the canonical orientation.

The CUDA backend's generic kernels decode these records inside stage 1; the
tensor-core paths expand V once at prepare time on the device
(``nqb_decode_product_codebook``) into their tile layout.  This module is the
host-side container.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from nanoquant_b200.backend import QuantizedLinearSpec
from nanoquant_b200.packed import (
    PACKED_LAYOUT_VERSION,
    PACKED_WORD_BITS,
    PackedLayerState,
    pack_sign_matrix,
    packed_word_count,
    unpack_sign_matrix,
)

PRODUCT_CODEBOOK_FORMAT_VERSION = "product-codebook-free-k16-v1"
PRODUCT_CODEBOOK_INDEX_BITS = 16
PRODUCT_CODEBOOK_HALF_BITS = 16
PRODUCT_CODEBOOK_HALF_INDEX_BITS = 8
PRODUCT_CODEBOOK_TABLE_SIZE = 1 << PRODUCT_CODEBOOK_HALF_INDEX_BITS


def product_codebook_payload_word_count(record_count: int) -> int:
    """int32 words holding ``record_count`` 16-bit records (reference product_codebook.py:33-36)."""

    if record_count <= 0:
        raise ValueError("product-codebook record count must be positive")
    return math.ceil(record_count * PRODUCT_CODEBOOK_INDEX_BITS / PACKED_WORD_BITS)


def pack_product_codebook_indices(indices: torch.Tensor) -> torch.Tensor:
    """Pack a row-major matrix of unsigned 16-bit records, two per word (reference :39-56)."""

    if (
        indices.ndim != 2
        or indices.numel() == 0
        or not indices.is_contiguous()
        or indices.dtype not in (torch.int16, torch.int32, torch.int64)
    ):
        raise ValueError("product-codebook indices must be a non-empty contiguous matrix")
    flat = indices.detach().to(device="cpu", dtype=torch.int64).reshape(-1).numpy()
    if bool(np.any(flat < 0)) or bool(np.any(flat >= 1 << 16)):
        raise ValueError("product-codebook index is outside the 16-bit range")
    halves = np.zeros(2 * product_codebook_payload_word_count(flat.size), dtype=np.uint16)
    halves[: flat.size] = flat.astype(np.uint16)
    return torch.from_numpy(halves.view("<i4").copy())


def unpack_product_codebook_indices(payload: torch.Tensor, shape: tuple[int, int]) -> torch.Tensor:
    """Decode the 16-bit record stream back to an int32 matrix (reference :59-81)."""

    if len(shape) != 2 or min(shape) <= 0:
        raise ValueError("product-codebook index shape must be positive")
    count = shape[0] * shape[1]
    words = product_codebook_payload_word_count(count)
    if payload.dtype != torch.int32 or tuple(payload.shape) != (words,) or not payload.is_contiguous():
        raise ValueError(f"product-codebook payload must be contiguous int32 with shape ({words},)")
    halves = np.ascontiguousarray(payload.detach().to("cpu").numpy()).view("<u2")
    if count % 2 and halves[-1] != 0:
        raise ValueError("product-codebook payload has a non-zero padding record")
    records = halves[:count].astype(np.int32).reshape(shape)
    return torch.from_numpy(np.ascontiguousarray(records)).to(payload.device)


def pack_product_half_table(signs: torch.Tensor) -> torch.Tensor:
    """Pack a 256x16 sign table into 256 int16 half-words, bit j = column j (reference :84-95)."""

    expected = (PRODUCT_CODEBOOK_TABLE_SIZE, PRODUCT_CODEBOOK_HALF_BITS)
    if tuple(signs.shape) != expected or not signs.is_contiguous():
        raise ValueError(f"product-codebook half table must have shape {expected}")
    host = signs.detach().to("cpu")
    if not bool(((host == 1) | (host == -1)).all()):
        raise ValueError("product-codebook half table contains a non-sign")
    bytes_ = np.packbits((host < 0).numpy(), axis=1, bitorder="little")
    return torch.from_numpy(np.ascontiguousarray(bytes_).view("<i2").reshape(-1).copy())


def unpack_product_half_table(words: torch.Tensor) -> torch.Tensor:
    """Expand 256 int16 half-words to a 256x16 +/-1 float table (reference :98-105)."""

    if words.dtype != torch.int16 or tuple(words.shape) != (PRODUCT_CODEBOOK_TABLE_SIZE,) or not words.is_contiguous():
        raise ValueError("product-codebook half table must be contiguous int16[256]")
    raw = np.ascontiguousarray(words.detach().to("cpu").numpy()).view(np.uint8).reshape(-1, 2)
    bits = np.unpackbits(raw, axis=1, bitorder="little")
    return torch.from_numpy((1.0 - 2.0 * bits.astype(np.float32)).copy())


def _half_words_u32(words: torch.Tensor) -> np.ndarray:
    return np.ascontiguousarray(words.detach().to("cpu").numpy()).view(np.uint16).astype(np.uint32)


def decode_product_codebook_right_words(
    free_right_words: torch.Tensor,
    coded_payload: torch.Tensor,
    first_half_words: torch.Tensor,
    second_half_words: torch.Tensor,
    *,
    rank: int,
    columns: int,
) -> torch.Tensor:
    """Expand a product-codebook right factor to layout-v1 words (reference :110-143)."""

    free_rows = int(free_right_words.shape[0])
    words_per_row = packed_word_count(columns)
    if (
        free_rows <= 0
        or free_rows >= rank
        or free_right_words.dtype != torch.int32
        or tuple(free_right_words.shape) != (free_rows, words_per_row)
        or not free_right_words.is_contiguous()
    ):
        raise ValueError("product-codebook free right-word prefix is invalid")
    coded_shape = (rank - free_rows, words_per_row)
    records = unpack_product_codebook_indices(coded_payload, coded_shape).to("cpu").numpy().astype(np.uint32)
    low = _half_words_u32(first_half_words)[records & 0xFF]
    high = _half_words_u32(second_half_words)[records >> 8]
    coded = (low | (high << 16)).astype(np.uint32).view(np.int32)
    result = np.concatenate((free_right_words.detach().to("cpu").numpy(), coded), axis=0)
    packed = torch.from_numpy(np.ascontiguousarray(result))
    unpack_sign_matrix(packed, rank, columns)  # canonical tail-padding check
    return packed


@dataclass(frozen=True, slots=True)
class ProductCodebookLayerState:
    """One product-codebook layer in factorisation orientation (reference :146-307)."""

    spec: QuantizedLinearSpec
    format: str
    factorization_transposed: bool
    free_rows: int
    factor_left_words: torch.Tensor
    factor_right_free_words: torch.Tensor
    factor_right_coded_payload: torch.Tensor
    first_half_words: torch.Tensor
    second_half_words: torch.Tensor
    factor_scale_pre: torch.Tensor
    factor_scale_mid: torch.Tensor
    factor_scale_post: torch.Tensor
    outlier_indices: torch.Tensor | None = None
    outlier_values: torch.Tensor | None = None
    outlier_scales: torch.Tensor | None = None

    def __post_init__(self) -> None:
        spec = self.spec
        if self.format != PRODUCT_CODEBOOK_FORMAT_VERSION:
            raise ValueError(f"unsupported product-codebook format: {self.format}")
        if spec.has_bias or spec.patch_rank:
            raise ValueError("product-codebook v1 does not carry optional bias or patches")
        if not 0 < self.free_rows < spec.rank:
            raise ValueError("product-codebook free rows must be between zero and rank")
        left_shape = (self.factor_out_features, packed_word_count(spec.rank))
        if (
            self.factor_left_words.dtype != torch.int32
            or tuple(self.factor_left_words.shape) != left_shape
            or not self.factor_left_words.is_contiguous()
        ):
            raise ValueError("product-codebook factor-left words differ")
        unpack_sign_matrix(self.factor_left_words, self.factor_out_features, spec.rank)
        unpack_product_half_table(self.first_half_words)
        unpack_product_half_table(self.second_half_words)
        decode_product_codebook_right_words(
            self.factor_right_free_words,
            self.factor_right_coded_payload,
            self.first_half_words,
            self.second_half_words,
            rank=spec.rank,
            columns=self.factor_in_features,
        )
        for name, value, size in (
            ("factor_scale_pre", self.factor_scale_pre, self.factor_in_features),
            ("factor_scale_mid", self.factor_scale_mid, spec.rank),
            ("factor_scale_post", self.factor_scale_post, self.factor_out_features),
        ):
            if (
                tuple(value.shape) != (size,)
                or not value.is_contiguous()
                or str(value.dtype).removeprefix("torch.") != spec.scale_dtype
                or not bool(torch.isfinite(value).all())
            ):
                raise ValueError(f"product-codebook {name} differs")
        if (self.outlier_indices is None) != (self.outlier_values is None):
            raise ValueError("product-codebook outlier tensors must be paired")
        if (self.outlier_indices is not None) != (spec.outlier_count > 0):
            raise ValueError("product-codebook outlier presence differs")
        self.to_packed()  # validates outliers through the packed container

    @property
    def factor_out_features(self) -> int:
        return self.spec.in_features if self.factorization_transposed else self.spec.out_features

    @property
    def factor_in_features(self) -> int:
        return self.spec.out_features if self.factorization_transposed else self.spec.in_features

    @property
    def coded_rows(self) -> int:
        return self.spec.rank - self.free_rows

    @property
    def record_count(self) -> int:
        return self.coded_rows * packed_word_count(self.factor_in_features)

    def decoded_right_words(self) -> torch.Tensor:
        """Factorisation-space right factor as layout-v1 words."""

        return decode_product_codebook_right_words(
            self.factor_right_free_words,
            self.factor_right_coded_payload,
            self.first_half_words,
            self.second_half_words,
            rank=self.spec.rank,
            columns=self.factor_in_features,
        )

    def to_packed(self) -> PackedLayerState:
        """Decode to the canonical packed layer (reference :229-269)."""

        spec = self.spec
        right_words = self.decoded_right_words()
        if self.factorization_transposed:
            factor_left = unpack_sign_matrix(self.factor_left_words, self.factor_out_features, spec.rank)
            factor_right = unpack_sign_matrix(right_words, spec.rank, self.factor_in_features)
            left_words = pack_sign_matrix(factor_right.mT.contiguous())
            right_words = pack_sign_matrix(factor_left.mT.contiguous())
            scale_pre, scale_post = self.factor_scale_post, self.factor_scale_pre
        else:
            left_words = self.factor_left_words
            scale_pre, scale_post = self.factor_scale_pre, self.factor_scale_post
        return PackedLayerState(
            spec,
            PACKED_LAYOUT_VERSION,
            left_words,
            right_words,
            scale_pre,
            self.factor_scale_mid,
            scale_post,
            outlier_indices=self.outlier_indices,
            outlier_values=self.outlier_values,
            outlier_scales=self.outlier_scales,
        )

    def compact_logical_bits(self) -> int:
        """Storage cost in bits, counted as the reference does (reference :271-295)."""

        spec = self.spec
        index_bits = math.ceil(math.log2(spec.in_features)) * spec.outlier_count
        value_bits = 8 if spec.outlier_value_dtype == "int8" else 16
        outlier_bits = spec.out_features * spec.outlier_count * value_bits
        outlier_scale_bits = spec.outlier_count * 16 if spec.has_outlier_scales else 0
        scale_count = self.factor_scale_pre.numel() + self.factor_scale_mid.numel() + self.factor_scale_post.numel()
        return (
            32 * self.factor_left_words.numel()
            + 32 * self.factor_right_free_words.numel()
            + PRODUCT_CODEBOOK_INDEX_BITS * self.record_count
            + 2 * PRODUCT_CODEBOOK_TABLE_SIZE * PRODUCT_CODEBOOK_HALF_BITS
            + 16
            + 16 * scale_count
            + index_bits
            + outlier_bits
            + outlier_scale_bits
        )


__all__ = [
    "PRODUCT_CODEBOOK_FORMAT_VERSION",
    "PRODUCT_CODEBOOK_HALF_BITS",
    "PRODUCT_CODEBOOK_HALF_INDEX_BITS",
    "PRODUCT_CODEBOOK_INDEX_BITS",
    "PRODUCT_CODEBOOK_TABLE_SIZE",
    "ProductCodebookLayerState",
    "decode_product_codebook_right_words",
    "pack_product_codebook_indices",
    "pack_product_half_table",
    "product_codebook_payload_word_count",
    "unpack_product_codebook_indices",
    "unpack_product_half_table",
]
