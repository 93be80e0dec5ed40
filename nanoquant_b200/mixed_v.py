"""Mixed free/codebook right factor (``mixed-v-free-k10-pair9-v1``).

Restates ``src/nanoquant/runtime/mixed_v.py:1-293`` of the reference.  A
layer keeps its first ``free_rows`` rows of ``V`` as plain layout-v1 words.
Every other word of ``V`` is one 19-bit record: bits 0..9 index a table of
1024 full sign words, bits 10..18 name one of the 496 bit pairs ``(a, b)``,
``a < b < 32`` (numbered in lexicographic order), whose two bits are flipped
in the table word.  Records are packed back to back, least significant bit
first, across consecutive int32 words; the unused tail bits are zero.

The CUDA backend expands the records once at prepare time on the device
(``nqb_decode_mixed_v``), as the reference's backend does
(``cuda_backend.py:209-224``), and then runs the layer as a packed layer.
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
    packed_word_count,
)

MIXED_V_FORMAT_VERSION = "mixed-v-free-k10-pair9-v1"
MIXED_V_INDEX_BITS = 10
MIXED_V_CORRECTION_BITS = 9
MIXED_V_RECORD_BITS = MIXED_V_INDEX_BITS + MIXED_V_CORRECTION_BITS
MIXED_V_CODEBOOK_SIZE = 1 << MIXED_V_INDEX_BITS
MIXED_V_CORRECTION_PAIR_COUNT = math.comb(PACKED_WORD_BITS, 2)

_BIT_WEIGHTS = np.left_shift(np.uint32(1), np.arange(MIXED_V_RECORD_BITS, dtype=np.uint32))


def mixed_v_payload_word_count(record_count: int) -> int:
    """int32 words holding ``record_count`` 19-bit records (reference mixed_v.py:25-28)."""

    if record_count <= 0:
        raise ValueError("mixed-V record count must be positive")
    return math.ceil(record_count * MIXED_V_RECORD_BITS / PACKED_WORD_BITS)


def _pair_bits() -> tuple[np.ndarray, np.ndarray]:
    first, second = np.triu_indices(PACKED_WORD_BITS, k=1)  # row-major: lexicographic (a, b), a < b
    return first.astype(np.int64), second.astype(np.int64)


def mixed_v_correction_pair_table(*, device: str | torch.device = "cpu") -> torch.Tensor:
    """Pair id -> ``a | b << 8`` as int32[512]; ids 496..511 hold 0 (reference mixed_v.py:31-45)."""

    first, second = _pair_bits()
    table = np.zeros(1 << MIXED_V_CORRECTION_BITS, dtype=np.int32)
    table[: first.size] = (first | (second << 8)).astype(np.int32)
    return torch.from_numpy(table).to(device)


def _check_fields(indices: torch.Tensor, pairs: torch.Tensor) -> None:
    if (
        indices.ndim != 2
        or tuple(indices.shape) != tuple(pairs.shape)
        or not indices.is_contiguous()
        or not pairs.is_contiguous()
        or indices.numel() == 0
    ):
        raise ValueError("mixed-V record fields must be matching non-empty contiguous matrices")
    for name, value in (("codebook indices", indices), ("correction pair ids", pairs)):
        if value.dtype not in (torch.int16, torch.int32, torch.int64):
            raise ValueError(f"mixed-V {name} must use an integer dtype")
    if bool(((indices < 0) | (indices >= MIXED_V_CODEBOOK_SIZE)).any()):
        raise ValueError("mixed-V codebook index is outside the 10-bit codebook")
    if bool(((pairs < 0) | (pairs >= MIXED_V_CORRECTION_PAIR_COUNT)).any()):
        raise ValueError("mixed-V correction pair id is outside the 496 valid pairs")


def pack_mixed_v_records(codebook_indices: torch.Tensor, correction_pair_ids: torch.Tensor) -> torch.Tensor:
    """Row-major ``(10-bit index, 9-bit pair)`` records -> minimal int32 stream (reference :48-71)."""

    _check_fields(codebook_indices, correction_pair_ids)
    index = codebook_indices.detach().to("cpu", torch.int64).reshape(-1).numpy().astype(np.uint32)
    pair = correction_pair_ids.detach().to("cpu", torch.int64).reshape(-1).numpy().astype(np.uint32)
    records = index | (pair << MIXED_V_INDEX_BITS)
    # the stream as bits, LSB-first per record, then LSB-first per word
    bits = ((records[:, None] & _BIT_WEIGHTS) != 0).astype(np.uint8).reshape(-1)
    words = mixed_v_payload_word_count(records.size)
    stream = np.zeros(words * PACKED_WORD_BITS, dtype=np.uint8)
    stream[: bits.size] = bits
    packed = np.packbits(stream, bitorder="little").view("<i4")
    return torch.from_numpy(packed.copy())


def unpack_mixed_v_records(payload: torch.Tensor, shape: tuple[int, int]) -> tuple[torch.Tensor, torch.Tensor]:
    """Decode and validate the minimal 19-bit stream -> (indices, pair ids) int32 (reference :74-101)."""

    if len(shape) != 2 or min(shape) <= 0:
        raise ValueError("mixed-V record shape must contain two positive dimensions")
    count = shape[0] * shape[1]
    words = mixed_v_payload_word_count(count)
    if payload.dtype != torch.int32 or tuple(payload.shape) != (words,) or not payload.is_contiguous():
        raise ValueError(f"mixed-V payload must be contiguous int32 with shape ({words},)")
    raw = np.ascontiguousarray(payload.detach().to("cpu").numpy()).view(np.uint8)
    bits = np.unpackbits(raw, bitorder="little")
    used = count * MIXED_V_RECORD_BITS
    if bool(bits[used:].any()):
        raise ValueError("mixed-V payload has a non-zero padding bit")
    records = (bits[:used].reshape(count, MIXED_V_RECORD_BITS).astype(np.uint32) * _BIT_WEIGHTS).sum(
        axis=1, dtype=np.uint32)
    indices = torch.from_numpy((records & (MIXED_V_CODEBOOK_SIZE - 1)).astype(np.int32).reshape(shape))
    pairs = torch.from_numpy((records >> MIXED_V_INDEX_BITS).astype(np.int32).reshape(shape))
    _check_fields(indices, pairs)
    return indices.to(payload.device), pairs.to(payload.device)


def decode_mixed_v_right_words(
    free_right_words: torch.Tensor,
    coded_payload: torch.Tensor,
    codebook_words: torch.Tensor,
    *,
    rank: int,
    in_features: int,
) -> torch.Tensor:
    """Expand a mixed-V right factor to layout-v1 words ``[rank, ceil(n/32)]`` (reference :104-123)."""

    free_rows = int(free_right_words.shape[0])
    words_per_row = packed_word_count(in_features)
    if not 0 < free_rows < rank:
        raise ValueError("mixed-V free row count must be between zero and rank")
    indices, pairs = unpack_mixed_v_records(coded_payload, (rank - free_rows, words_per_row))
    first, second = _pair_bits()
    flips = ((np.uint64(1) << first.astype(np.uint64)) | (np.uint64(1) << second.astype(np.uint64))).astype(np.uint32)
    book = np.ascontiguousarray(codebook_words.detach().to("cpu").numpy()).view(np.uint32)
    coded = book[indices.to("cpu").numpy()] ^ flips[pairs.to("cpu").numpy()]
    free = free_right_words.detach().to("cpu").numpy()
    words = np.concatenate((free, coded.view(np.int32)), axis=0)
    return torch.from_numpy(np.ascontiguousarray(words)).to(free_right_words.device)


@dataclass(frozen=True, slots=True)
class MixedVLayerState:
    """A packed layer whose V tail holds one 19-bit record per canonical word (reference :126-196)."""

    spec: QuantizedLinearSpec
    format: str
    free_rows: int
    left_words: torch.Tensor
    free_right_words: torch.Tensor
    coded_payload: torch.Tensor
    codebook_words: torch.Tensor
    scale_pre: torch.Tensor
    scale_mid: torch.Tensor
    scale_post: torch.Tensor
    bias: torch.Tensor | None = None
    outlier_indices: torch.Tensor | None = None
    outlier_values: torch.Tensor | None = None
    outlier_scales: torch.Tensor | None = None
    patch_left: torch.Tensor | None = None
    patch_right: torch.Tensor | None = None

    def __post_init__(self) -> None:
        if self.format != MIXED_V_FORMAT_VERSION:
            raise ValueError(f"unsupported mixed-V format: {self.format}")
        if not 0 < self.free_rows < self.spec.rank:
            raise ValueError("mixed-V free row count must be between zero and rank")
        words_per_row = packed_word_count(self.spec.in_features)
        if tuple(self.free_right_words.shape) != (self.free_rows, words_per_row):
            raise ValueError("mixed-V free right-word shape differs")
        if self.free_right_words.dtype != torch.int32 or not self.free_right_words.is_contiguous():
            raise ValueError("mixed-V free right words must be contiguous int32")
        if tuple(self.codebook_words.shape) != (MIXED_V_CODEBOOK_SIZE,):
            raise ValueError("mixed-V codebook must contain exactly 1024 words")
        if self.codebook_words.dtype != torch.int32 or not self.codebook_words.is_contiguous():
            raise ValueError("mixed-V codebook words must be contiguous int32")
        # payload, pair ids, sign padding, scales and sidecars: through the packed container
        self.to_packed()

    @property
    def coded_rows(self) -> int:
        return self.spec.rank - self.free_rows

    @property
    def record_count(self) -> int:
        return self.coded_rows * packed_word_count(self.spec.in_features)

    def to_packed(self) -> PackedLayerState:
        right_words = decode_mixed_v_right_words(
            self.free_right_words, self.coded_payload, self.codebook_words,
            rank=self.spec.rank, in_features=self.spec.in_features)
        return PackedLayerState(
            self.spec, PACKED_LAYOUT_VERSION, self.left_words, right_words, self.scale_pre, self.scale_mid,
            self.scale_post, self.bias, self.outlier_indices, self.outlier_values, self.outlier_scales,
            self.patch_left, self.patch_right)

    def to_logical(self):  # type: ignore[no-untyped-def]
        return self.to_packed().to_logical()


def mixed_v_from_packed_words(
    packed: PackedLayerState,
    *,
    free_rows: int,
    codebook_words: torch.Tensor,
    codebook_indices: torch.Tensor,
    correction_pair_ids: torch.Tensor,
) -> MixedVLayerState:
    """Compact state from exact coded-tail records of ``packed`` (reference :199-237)."""

    expected = (packed.spec.rank - free_rows, packed_word_count(packed.spec.in_features))
    if tuple(codebook_indices.shape) != expected or tuple(correction_pair_ids.shape) != expected:
        raise ValueError(f"mixed-V coded record matrices must have shape {expected}")
    state = MixedVLayerState(
        packed.spec, MIXED_V_FORMAT_VERSION, free_rows, packed.left_words,
        packed.right_words[:free_rows].contiguous(), pack_mixed_v_records(codebook_indices, correction_pair_ids),
        codebook_words.detach().cpu().to(torch.int32).contiguous(), packed.scale_pre, packed.scale_mid,
        packed.scale_post, packed.bias, packed.outlier_indices, packed.outlier_values, packed.outlier_scales,
        packed.patch_left, packed.patch_right)
    if not torch.equal(state.to_packed().right_words.cpu(), packed.right_words.cpu()):
        raise ValueError("mixed-V records do not reconstruct the supplied packed right factor")
    return state


__all__ = [
    "MIXED_V_CODEBOOK_SIZE",
    "MIXED_V_CORRECTION_BITS",
    "MIXED_V_CORRECTION_PAIR_COUNT",
    "MIXED_V_FORMAT_VERSION",
    "MIXED_V_INDEX_BITS",
    "MIXED_V_RECORD_BITS",
    "MixedVLayerState",
    "decode_mixed_v_right_words",
    "mixed_v_correction_pair_table",
    "mixed_v_from_packed_words",
    "mixed_v_payload_word_count",
    "pack_mixed_v_records",
    "unpack_mixed_v_records",
]
