"""Int8 residual output-row overlay for a packed layer.

A small set of output rows ``o = row_ids[j]`` carries a dense int8 residual
row ``R[j, :]`` with one scale per row, so that

    y[t, o] += scale[j] * sum_i R[j, i] * x[t, i]

on top of the packed low-rank product.  This is the row form of the outlier
sidecar: the reference runtime only carries outliers as salient input
*columns* (``src/nanoquant/runtime/packed.py:230-352``); its cost model for
residual rows lives in ``src/nanoquant/domain/structured_sidecar.py:32-118``
but it has no runtime type for them, so this container is new.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from nanoquant_b200.mixed_v import MixedVLayerState
from nanoquant_b200.packed import PackedLayerState
from nanoquant_b200.product_codebook import ProductCodebookLayerState

_SCALE_DTYPES = (torch.float16, torch.bfloat16, torch.float32)


@dataclass(frozen=True, slots=True)
class OutlierRowOverlay:
    """Residual int8 rows: ``row_ids`` [R] int32 ascending, ``values`` [R, in], ``scales`` [R]."""

    row_ids: torch.Tensor
    values: torch.Tensor
    scales: torch.Tensor

    def validate(self, out_features: int, in_features: int) -> None:
        rows = int(self.row_ids.shape[0]) if self.row_ids.ndim == 1 else -1
        if self.row_ids.dtype != torch.int32 or self.row_ids.ndim != 1 or not self.row_ids.is_contiguous():
            raise ValueError("overlay row ids must be a contiguous int32 vector")
        if rows <= 0 or rows > out_features:
            raise ValueError("overlay row count is outside the output dimension")
        ids = self.row_ids.to(torch.int64)
        if bool((ids < 0).any()) or bool((ids >= out_features).any()):
            raise ValueError("overlay row id is outside the output dimension")
        if not bool((ids[1:] > ids[:-1]).all()):
            raise ValueError("overlay row ids must be strictly increasing")
        if self.values.dtype != torch.int8 or tuple(self.values.shape) != (rows, in_features):
            raise ValueError("overlay values must be int8 with shape [rows, in_features]")
        if not self.values.is_contiguous():
            raise ValueError("overlay values must be contiguous")
        if self.scales.dtype not in _SCALE_DTYPES or tuple(self.scales.shape) != (rows,):
            raise ValueError("overlay scales must be one float per row")
        if not self.scales.is_contiguous() or not bool(torch.isfinite(self.scales).all()):
            raise ValueError("overlay scales must be contiguous and finite")


@dataclass(frozen=True, slots=True)
class OverlaidLayerState:
    """A packed or product-codebook layer plus an int8 residual-row overlay."""

    base: PackedLayerState | ProductCodebookLayerState | MixedVLayerState
    overlay: OutlierRowOverlay

    def __post_init__(self) -> None:
        if not isinstance(self.base, (PackedLayerState, ProductCodebookLayerState, MixedVLayerState)):
            raise TypeError("overlay base must be a PackedLayerState, ProductCodebookLayerState or MixedVLayerState")
        self.overlay.validate(self.spec.out_features, self.spec.in_features)

    @property
    def spec(self):  # type: ignore[no-untyped-def]
        return self.base.spec


__all__ = ["OutlierRowOverlay", "OverlaidLayerState"]
