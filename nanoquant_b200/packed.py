"""NanoQuant packed layout v1: sign words and the validated packed layer state.

Layout v1 (reference ``src/nanoquant/runtime/packed.py:84-218`` and
``Docs/19-nanoquant-packed-layout-v1.md``) stores a +/-1 matrix row by row in
int32 words: column ``c`` lives in word ``c // 32`` at bit ``c % 32``, least
significant bit first; a set bit means -1, a clear bit +1, and the unused tail
bits of the last word of every row are zero.  ``U`` (left, ``[out, rank]``) is
packed along rank and ``V`` (right, ``[rank, in]``) along the input features.

The pack/unpack routines here are written with numpy bit packing; they must be
bit-identical to the reference, which the golden fixtures check.
"""

from __future__ import annotations

from collections.abc import Iterator
from contextlib import contextmanager
from contextvars import ContextVar
from dataclasses import dataclass

import numpy as np
import torch

from nanoquant_b200.backend import QuantizedLinearSpec
from nanoquant_b200.logical import LogicalLayerState, canonical_torch_dtype, parse_torch_dtype

PACKED_LAYOUT_VERSION = "llama.cpp-i32-lsb-v1"
PACKED_WORD_BITS = 32
PACKED_WORD_DTYPE = "int32"
PACKED_TENSOR_NAMESPACE = f"layouts.{PACKED_LAYOUT_VERSION}"

# Sidecar tensor names used by the GGUF export of layout v1 (reference packed.py:35-45).
# They are a wire format shared with llama.cpp, so they are kept verbatim.
GGUF_TENSOR_SUFFIXES = (
    ("factor_right_words", "nq_v"),
    ("factor_left_words", "nq_u"),
    ("scale_pre", "nq_scale_pre"),
    ("scale_mid", "nq_scale_mid"),
    ("scale_post", "nq_scale_post"),
    ("outlier_indices", "nq_salient_idx"),
    ("outlier_values", "nq_salient_weight"),
    ("outlier_scales", "nq_salient_scale"),
    ("bias", "bias"),
)


@dataclass(frozen=True, slots=True)
class PackedLayoutMetadata:
    """Facts about layout v1 that a consumer may check (reference packed.py:84-136)."""

    version: str = PACKED_LAYOUT_VERSION
    word_dtype: str = PACKED_WORD_DTYPE
    word_bits: int = PACKED_WORD_BITS
    bit_order: str = "least-significant-bit-first"
    positive_bit: int = 0
    negative_bit: int = 1
    padding_bit: int = 0
    minimum_alignment_bytes: int = 4
    vector_alignment_bytes: int = 16
    tensor_namespace: str = PACKED_TENSOR_NAMESPACE
    bias_storage: str = "separate-additive-tensor"

    def __post_init__(self) -> None:
        if self.version != PACKED_LAYOUT_VERSION:
            raise ValueError(f"unsupported packed layout version: {self.version}")
        if (self.word_dtype, self.word_bits) != (PACKED_WORD_DTYPE, PACKED_WORD_BITS):
            raise ValueError("packed layout word representation differs from the runtime")
        if self.bit_order != "least-significant-bit-first":
            raise ValueError("packed layout bit order differs from the runtime")
        if (self.positive_bit, self.negative_bit, self.padding_bit) != (0, 1, 0):
            raise ValueError("packed layout sign or padding encoding differs from the runtime")


def packed_word_count(columns: int) -> int:
    """Words per packed row (reference packed.py:139-142)."""

    if columns <= 0:
        raise ValueError("packed sign column count must be positive")
    return -(-columns // PACKED_WORD_BITS)


def packed_row_stride_bytes(columns: int) -> int:
    """Byte stride between packed rows (reference packed.py:145-146)."""

    return 4 * packed_word_count(columns)


def supports_vector_word_loads(words: torch.Tensor) -> bool:
    """True when every row of ``words`` starts on a 16-byte boundary (reference packed.py:149-158)."""

    return (
        words.ndim == 2
        and words.dtype == torch.int32
        and words.is_contiguous()
        and words.data_ptr() % 16 == 0
        and (words.stride(0) * words.element_size()) % 16 == 0
    )


def _sign_matrix_numpy(signs: torch.Tensor) -> np.ndarray:
    if signs.ndim != 2 or not signs.is_contiguous():
        raise ValueError("logical signs must be a contiguous matrix")
    if signs.shape[0] <= 0 or signs.shape[1] <= 0:
        raise ValueError("logical sign matrix dimensions must be positive")
    host = signs.detach().to("cpu")
    if not bool(((host == 1) | (host == -1)).all()):
        raise ValueError("logical signs contain a value other than -1 or +1")
    return (host < 0).numpy()


def pack_sign_matrix(signs: torch.Tensor) -> torch.Tensor:
    """Pack a +/-1 matrix into layout-v1 int32 words (reference packed.py:170-188).

    Returns a contiguous CPU int32 tensor of shape ``[rows, ceil(cols / 32)]``.
    """

    negative = _sign_matrix_numpy(signs)
    rows, columns = negative.shape
    words = packed_word_count(columns)
    padded = np.zeros((rows, words * PACKED_WORD_BITS), dtype=np.bool_)
    padded[:, :columns] = negative
    # little-endian bit order within each byte, bytes in little-endian word order
    as_bytes = np.packbits(padded, axis=1, bitorder="little")
    packed = np.ascontiguousarray(as_bytes).view("<i4").reshape(rows, words)
    return torch.from_numpy(packed.astype(np.int32, copy=True))


def _check_packed_matrix(words: torch.Tensor, rows: int, columns: int) -> None:
    expected = (rows, packed_word_count(columns))
    if words.dtype != torch.int32 or tuple(words.shape) != expected or not words.is_contiguous():
        raise ValueError(
            f"packed sign matrix must be contiguous int32 with shape {expected}, got "
            f"{words.dtype} {tuple(words.shape)}"
        )
    tail = columns % PACKED_WORD_BITS
    if tail:
        padding_mask = -(1 << tail)  # bits tail..31 of an int32 word
        _value_check((words[:, -1].detach() & padding_mask).ne(0).any(),
                     "packed sign matrix has a non-zero padding bit")


def unpack_sign_matrix(
    words: torch.Tensor,
    rows: int,
    columns: int,
    *,
    dtype: torch.dtype = torch.float32,
) -> torch.Tensor:
    """Expand layout-v1 words back to a dense +/-1 matrix (reference packed.py:204-218)."""

    _check_packed_matrix(words, rows, columns)
    host = np.ascontiguousarray(words.detach().to("cpu").numpy()).view(np.uint8)
    bits = np.unpackbits(host.reshape(rows, -1), axis=1, bitorder="little")[:, :columns]
    signs = 1.0 - 2.0 * bits.astype(np.float32)
    return torch.from_numpy(np.ascontiguousarray(signs)).to(dtype=dtype).to(words.device).contiguous()


def _factor_dtype(name: str) -> torch.dtype:
    if name not in ("float16", "bfloat16", "float32"):
        raise ValueError(f"packed layout does not support logical factor dtype: {name}")
    return parse_torch_dtype(name)


# Value checks (padding bits, finiteness, salient-index order) read tensor
# contents.  Outside `deferred_value_checks` each one raises at once, which
# costs a device synchronisation per check for device tensors; inside it they
# are recorded as 0-dim flags and evaluated together when the block exits.
_DEFERRED: ContextVar[list[tuple[torch.Tensor, str]] | None] = ContextVar("nanoquant_b200_deferred_checks",
                                                                          default=None)


def _value_check(failed: torch.Tensor, message: str) -> None:
    pending = _DEFERRED.get()
    if pending is None:
        if bool(failed):
            raise ValueError(message)
    else:
        pending.append((failed.reshape(()), message))


@contextmanager
def deferred_value_checks() -> Iterator[None]:
    """Defer the value checks of the packed layers constructed in the block.

    Shape, dtype and presence checks still raise at construction.  At exit the
    recorded flags are copied to the host in one transfer per device and the
    first failed check, in construction order, raises its ``ValueError``.
    """

    pending: list[tuple[torch.Tensor, str]] = []
    token = _DEFERRED.set(pending)
    try:
        yield
    finally:
        _DEFERRED.reset(token)
    if not pending:
        return
    failed = [False] * len(pending)
    by_device: dict[torch.device, list[int]] = {}
    for index, (flag, _) in enumerate(pending):
        by_device.setdefault(flag.device, []).append(index)
    for device, indices in by_device.items():
        values = torch.stack([pending[i][0] for i in indices]).to("cpu")
        for i, value in zip(indices, values.tolist(), strict=True):
            failed[i] = bool(value)
    for (_, message), bad in zip(pending, failed, strict=True):
        if bad:
            raise ValueError(message)


def _require_finite(value: torch.Tensor, message: str) -> None:
    _value_check(~torch.isfinite(value).all(), message)


@dataclass(frozen=True, slots=True)
class PackedLayerState:
    """Validated packed layer (reference packed.py:230-382).

    ``left_words`` is ``U`` packed along rank, ``right_words`` is ``V`` packed
    along the input features; the three scales share ``spec.scale_dtype``.
    """

    spec: QuantizedLinearSpec
    layout: str
    left_words: torch.Tensor
    right_words: torch.Tensor
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
        spec = self.spec
        if self.layout != PACKED_LAYOUT_VERSION:
            raise ValueError(f"unsupported packed layer layout: {self.layout}")
        _check_packed_matrix(self.left_words, spec.out_features, spec.rank)
        _check_packed_matrix(self.right_words, spec.rank, spec.in_features)
        for name, value, size in (
            ("scale_pre", self.scale_pre, spec.in_features),
            ("scale_mid", self.scale_mid, spec.rank),
            ("scale_post", self.scale_post, spec.out_features),
        ):
            if tuple(value.shape) != (size,) or not value.is_contiguous():
                raise ValueError(f"packed layer {name} shape or layout differs")
            if canonical_torch_dtype(value.dtype) != spec.scale_dtype:
                raise ValueError(f"packed layer {name} dtype differs")
            _require_finite(value, f"packed layer {name} contains a non-finite value")
        self._check_bias()
        self._check_outliers()
        self._check_patch()

    def _check_bias(self) -> None:
        spec = self.spec
        if (self.bias is not None) != spec.has_bias:
            raise ValueError("packed layer bias presence differs from its specification")
        if self.bias is None:
            return
        if tuple(self.bias.shape) != (spec.out_features,) or not self.bias.is_contiguous():
            raise ValueError("packed layer bias shape differs")
        if canonical_torch_dtype(self.bias.dtype) != (spec.bias_dtype or spec.scale_dtype):
            raise ValueError("packed layer bias dtype differs")
        _require_finite(self.bias, "packed layer bias contains a non-finite value")

    def _check_outliers(self) -> None:
        spec = self.spec
        indices, values, scales = self.outlier_indices, self.outlier_values, self.outlier_scales
        if (indices is None) != (values is None):
            raise ValueError("packed layer outlier indices and values must be paired")
        if (indices is not None) != (spec.outlier_count > 0):
            raise ValueError("packed layer outlier presence differs from its specification")
        if indices is not None and values is not None:
            if indices.dtype != torch.int32:
                raise ValueError("packed llama.cpp salient indices must be int32")
            if tuple(indices.shape) != (spec.outlier_count,) or not indices.is_contiguous():
                raise ValueError("packed layer outlier index shape differs")
            if tuple(values.shape) != (spec.out_features, spec.outlier_count) or not values.is_contiguous():
                raise ValueError("packed layer outlier value shape differs")
            if canonical_torch_dtype(values.dtype) != spec.outlier_value_dtype:
                raise ValueError("packed layer outlier value dtype differs")
            positions = indices.to(torch.int64)
            _value_check(((positions < 0) | (positions >= spec.in_features)).any(),
                         "packed layer outlier index is outside the input dimension")
            _value_check(~(positions[1:] > positions[:-1]).all(),
                         "packed layer outlier indices must be strictly increasing")
            # The kernels add salient columns on a separate path, so their pre-scale
            # must be exactly zero (reference packed.py:303-307).  (Clamped so that
            # a deferred check never indexes out of range.)
            safe = positions.clamp(0, spec.in_features - 1).to(self.scale_pre.device)
            _value_check((self.scale_pre.index_select(0, safe) != 0).any(),
                         "packed llama.cpp salient columns require exactly zero scale_pre entries")
            if values.dtype not in (torch.int8, torch.float16, torch.bfloat16, torch.float32):
                raise ValueError("packed llama.cpp salient value dtype is unsupported")
            if values.is_floating_point():
                _require_finite(values, "packed layer outlier value contains a non-finite value")
        if (scales is not None) != spec.has_outlier_scales:
            raise ValueError("packed layer outlier scale presence differs")
        if scales is not None:
            if values is None or values.dtype != torch.int8:
                raise ValueError("packed llama.cpp salient scales require int8 values")
            if tuple(scales.shape) != (spec.outlier_count,) or not scales.is_contiguous():
                raise ValueError("packed llama.cpp salient scales must have one value per column")
            if canonical_torch_dtype(scales.dtype) != spec.scale_dtype:
                raise ValueError("packed layer outlier scale dtype differs")
            _require_finite(scales, "packed layer outlier scale contains a non-finite value")
        if values is not None and values.dtype == torch.int8 and scales is None:
            raise ValueError("packed llama.cpp int8 salient values require scales")

    def _check_patch(self) -> None:
        spec = self.spec
        left, right = self.patch_left, self.patch_right
        if (left is None) != (right is None):
            raise ValueError("packed low-rank patch tensors must be paired")
        if (left is not None) != (spec.patch_rank > 0):
            raise ValueError("packed patch presence differs from its specification")
        if left is None or right is None:
            return
        if tuple(left.shape) != (spec.out_features, spec.patch_rank):
            raise ValueError("packed patch-left shape differs")
        if tuple(right.shape) != (spec.patch_rank, spec.in_features):
            raise ValueError("packed patch-right shape differs")
        if not (left.is_contiguous() and right.is_contiguous()):
            raise ValueError("packed low-rank patch tensors must be contiguous")
        for value in (left, right):
            if canonical_torch_dtype(value.dtype) != spec.patch_value_dtype:
                raise ValueError("packed patch dtype differs")
            _require_finite(value, "packed low-rank patch contains a non-finite value")

    def to_logical(self) -> LogicalLayerState:
        """Unpack both factors to dense +/-1 in ``spec.factor_dtype`` (reference packed.py:354-382)."""

        spec = self.spec
        factor = _factor_dtype(spec.factor_dtype)
        return LogicalLayerState(
            spec,
            unpack_sign_matrix(self.left_words, spec.out_features, spec.rank, dtype=factor),
            unpack_sign_matrix(self.right_words, spec.rank, spec.in_features, dtype=factor),
            self.scale_pre,
            self.scale_mid,
            self.scale_post,
            self.bias,
            self.outlier_indices,
            self.outlier_values,
            self.outlier_scales,
            self.patch_left,
            self.patch_right,
        )


def _host_copy(value: torch.Tensor | None) -> torch.Tensor | None:
    return None if value is None else value.detach().to("cpu").clone().contiguous()


def pack_logical_layer(state: LogicalLayerState) -> PackedLayerState:
    """Pack a dense logical layer into layout v1 (reference packed.py:393-411)."""

    indices = _host_copy(state.outlier_indices)
    return PackedLayerState(
        state.spec,
        PACKED_LAYOUT_VERSION,
        pack_sign_matrix(state.left_binary),
        pack_sign_matrix(state.right_binary),
        _host_copy(state.scale_pre),
        _host_copy(state.scale_mid),
        _host_copy(state.scale_post),
        _host_copy(state.bias),
        None if indices is None else indices.to(torch.int32),
        _host_copy(state.outlier_values),
        _host_copy(state.outlier_scales),
        _host_copy(state.patch_left),
        _host_copy(state.patch_right),
    )


__all__ = [
    "GGUF_TENSOR_SUFFIXES",
    "PACKED_LAYOUT_VERSION",
    "PACKED_TENSOR_NAMESPACE",
    "PACKED_WORD_BITS",
    "PACKED_WORD_DTYPE",
    "PackedLayerState",
    "PackedLayoutMetadata",
    "deferred_value_checks",
    "pack_logical_layer",
    "pack_sign_matrix",
    "packed_row_stride_bytes",
    "packed_word_count",
    "supports_vector_word_loads",
    "unpack_sign_matrix",
]
