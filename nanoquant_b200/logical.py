"""Dense +/-1 logical layer state and runtime dtype names.

Restates ``src/nanoquant/runtime/logical.py:1-149`` of the reference: the
canonical dtype spelling used by specs and capability tables, and the validated
dense-factor container that layout v1 packing starts from.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from nanoquant_b200.backend import QuantizedLinearSpec

# Canonical runtime dtype spellings (reference logical.py:11-20).
_NAME_TO_DTYPE: dict[str, torch.dtype] = {
    "float16": torch.float16,
    "bfloat16": torch.bfloat16,
    "float32": torch.float32,
    "int8": torch.int8,
    "int16": torch.int16,
    "int32": torch.int32,
    "int64": torch.int64,
    "uint8": torch.uint8,
}
_DTYPE_TO_NAME = {dtype: name for name, dtype in _NAME_TO_DTYPE.items()}


def parse_torch_dtype(name: str) -> torch.dtype:
    """Map a canonical runtime dtype name to a torch dtype (reference logical.py:23-29)."""

    if name not in _NAME_TO_DTYPE:
        raise ValueError(f"unsupported runtime tensor dtype: {name}")
    return _NAME_TO_DTYPE[name]


def canonical_torch_dtype(dtype: torch.dtype) -> str:
    """Map a torch dtype to its canonical runtime name (reference logical.py:32-38)."""

    if dtype not in _DTYPE_TO_NAME:
        raise ValueError(f"unsupported runtime tensor dtype: {dtype}")
    return _DTYPE_TO_NAME[dtype]


def _all_finite(value: torch.Tensor) -> bool:
    return bool(torch.isfinite(value).all())


def _is_sign_matrix(value: torch.Tensor) -> bool:
    return bool(((value == 1) | (value == -1)).all())


@dataclass(frozen=True, slots=True)
class LogicalLayerState:
    """Dense +/-1 factors plus scales and sidecars (reference logical.py:41-149)."""

    spec: QuantizedLinearSpec
    left_binary: torch.Tensor
    right_binary: torch.Tensor
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
        shaped = (
            ("left_binary", self.left_binary, (spec.out_features, spec.rank)),
            ("right_binary", self.right_binary, (spec.rank, spec.in_features)),
            ("scale_pre", self.scale_pre, (spec.in_features,)),
            ("scale_mid", self.scale_mid, (spec.rank,)),
            ("scale_post", self.scale_post, (spec.out_features,)),
        )
        for name, value, expected in shaped:
            if tuple(value.shape) != expected:
                raise ValueError(f"runtime tensor {name} has shape {tuple(value.shape)}, expected {expected}")
            if not value.is_contiguous():
                raise ValueError(f"runtime tensor {name} must be contiguous")
        if canonical_torch_dtype(self.left_binary.dtype) != spec.factor_dtype:
            raise ValueError("runtime left factor dtype differs from its specification")
        if self.right_binary.dtype != self.left_binary.dtype:
            raise ValueError("runtime factor dtypes differ")
        scales = (self.scale_pre, self.scale_mid, self.scale_post)
        if any(canonical_torch_dtype(value.dtype) != spec.scale_dtype for value in scales):
            raise ValueError("runtime scale dtype differs from its specification")
        if not all(_all_finite(value) for value in scales):
            raise ValueError("runtime scale contains a non-finite value")
        if not _is_sign_matrix(self.left_binary):
            raise ValueError("runtime left factor contains a value other than -1 or +1")
        if not _is_sign_matrix(self.right_binary):
            raise ValueError("runtime right factor contains a value other than -1 or +1")
        self._check_bias()
        self._check_outliers()
        self._check_patch()

    def _check_bias(self) -> None:
        spec = self.spec
        if (self.bias is not None) != spec.has_bias:
            raise ValueError("runtime bias presence differs from its specification")
        if self.bias is None:
            return
        if tuple(self.bias.shape) != (spec.out_features,):
            raise ValueError("runtime bias shape differs from the output dimension")
        if canonical_torch_dtype(self.bias.dtype) != (spec.bias_dtype or spec.scale_dtype):
            raise ValueError("runtime bias dtype differs from its specification")
        if not _all_finite(self.bias):
            raise ValueError("runtime bias contains a non-finite value")

    def _check_outliers(self) -> None:
        spec = self.spec
        present = self.outlier_indices is not None or self.outlier_values is not None
        if present != (spec.outlier_count > 0):
            raise ValueError("runtime outlier presence differs from its specification")
        if (self.outlier_indices is None) != (self.outlier_values is None):
            raise ValueError("runtime outlier indices and values must be provided together")
        if self.outlier_indices is not None and self.outlier_values is not None:
            if tuple(self.outlier_indices.shape) != (spec.outlier_count,):
                raise ValueError("runtime outlier index shape differs from its specification")
            if tuple(self.outlier_values.shape) != (spec.out_features, spec.outlier_count):
                raise ValueError("runtime outlier value shape differs from its specification")
            if self.outlier_indices.dtype not in (torch.int32, torch.int64):
                raise ValueError("runtime outlier indices must be int32 or int64")
            positions = self.outlier_indices.to(torch.int64)
            if bool((positions < 0).any()) or bool((positions >= spec.in_features).any()):
                raise ValueError("runtime outlier index is outside the input dimension")
            if not bool((positions[1:] > positions[:-1]).all()):
                raise ValueError("runtime outlier indices must be strictly increasing")
            if canonical_torch_dtype(self.outlier_values.dtype) != spec.outlier_value_dtype:
                raise ValueError("runtime outlier value dtype differs from its specification")
            if self.outlier_values.is_floating_point() and not _all_finite(self.outlier_values):
                raise ValueError("runtime outlier value contains a non-finite value")
        if (self.outlier_scales is not None) != spec.has_outlier_scales:
            raise ValueError("runtime outlier scale presence differs from its specification")
        if self.outlier_scales is not None:
            allowed = {(), (spec.outlier_count,), (spec.out_features, 1), (spec.out_features, spec.outlier_count)}
            if tuple(self.outlier_scales.shape) not in allowed:
                raise ValueError("runtime outlier scale shape is not broadcastable to outlier values")
            if canonical_torch_dtype(self.outlier_scales.dtype) != spec.scale_dtype:
                raise ValueError("runtime outlier scale dtype differs from the scale dtype")
            if not _all_finite(self.outlier_scales):
                raise ValueError("runtime outlier scale contains a non-finite value")

    def _check_patch(self) -> None:
        spec = self.spec
        if (self.patch_left is None) != (self.patch_right is None):
            raise ValueError("runtime low-rank patch tensors must be paired")
        if (self.patch_left is not None) != (spec.patch_rank > 0):
            raise ValueError("runtime patch presence differs from its specification")
        if self.patch_left is None or self.patch_right is None:
            return
        if tuple(self.patch_left.shape) != (spec.out_features, spec.patch_rank):
            raise ValueError("runtime patch-left shape differs from its specification")
        if tuple(self.patch_right.shape) != (spec.patch_rank, spec.in_features):
            raise ValueError("runtime patch-right shape differs from its specification")
        if not (self.patch_left.is_contiguous() and self.patch_right.is_contiguous()):
            raise ValueError("runtime low-rank patch tensors must be contiguous")
        for value in (self.patch_left, self.patch_right):
            if canonical_torch_dtype(value.dtype) != spec.patch_value_dtype:
                raise ValueError("runtime patch dtype differs from its specification")
            if not _all_finite(value):
                raise ValueError("runtime low-rank patch contains a non-finite value")


__all__ = ["LogicalLayerState", "canonical_torch_dtype", "parse_torch_dtype"]
