"""Operator contract for the packed binary low-rank linear.

This module restates the runtime backend boundary of NanoQuant's deployment
runtime (``src/nanoquant/runtime/backend.py:14-266`` in the reference) so that a
caller written against that boundary can hand its layers to this package
unchanged: the same dataclass names, field order, defaults, validation rules,
``NQ-INF-*`` rejection codes and check order.

Only the contract lives here.  The executing backend is
:class:`nanoquant_b200.cuda_backend.CudaPackedSm100Backend`.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Literal, Protocol, TypeAlias, runtime_checkable

import torch

DeviceLike: TypeAlias = str | torch.device
WorkloadKind: TypeAlias = Literal["prefill", "decode"]


def _canonical_dotted_name(name: str) -> bool:
    return bool(name) and not name.startswith("/") and ".." not in name.split(".")


@dataclass(frozen=True, slots=True)
class ProjectionMemberSpec:
    """One member slice of a grouped projection (reference ``backend.py:14-24``)."""

    name: str
    row_start: int
    row_end: int

    def __post_init__(self) -> None:
        if not _canonical_dotted_name(self.name):
            raise ValueError("runtime projection member name must be canonical")
        if self.row_start < 0 or self.row_end <= self.row_start:
            raise ValueError("runtime projection member slice must be non-empty")


@dataclass(frozen=True, slots=True)
class QuantizedLinearSpec:
    """Backend-independent description of one frozen linear (reference ``backend.py:27-73``)."""

    name: str
    logical_format: str
    in_features: int
    out_features: int
    rank: int
    factor_dtype: str
    scale_dtype: str
    outlier_count: int = 0
    outlier_value_dtype: str | None = None
    has_outlier_scales: bool = False
    has_bias: bool = False
    members: tuple[ProjectionMemberSpec, ...] = ()
    patch_rank: int = 0
    patch_value_dtype: str | None = None
    bias_dtype: str | None = None

    def __post_init__(self) -> None:
        if not _canonical_dotted_name(self.name):
            raise ValueError("runtime layer name must be a canonical dotted path")
        if min(self.in_features, self.out_features, self.rank) <= 0:
            raise ValueError("runtime linear dimensions and rank must be positive")
        if not 0 <= self.outlier_count <= self.in_features:
            raise ValueError("runtime outlier count is outside the input dimension")
        if (self.outlier_count > 0) != (self.outlier_value_dtype is not None):
            raise ValueError("runtime outlier dtype must be present exactly when outliers are present")
        if self.has_outlier_scales and self.outlier_count == 0:
            raise ValueError("runtime outlier scales require outlier values")
        if not 0 <= self.patch_rank <= min(self.in_features, self.out_features):
            raise ValueError("runtime patch rank is outside the linear dimensions")
        if (self.patch_rank > 0) != (self.patch_value_dtype is not None):
            raise ValueError("runtime patch dtype must be present exactly when a patch is present")
        if self.bias_dtype is not None and not self.has_bias:
            raise ValueError("runtime bias dtype requires a bias")
        if self.members:
            names = [member.name for member in self.members]
            if len(names) < 2 or len(set(names)) != len(names):
                raise ValueError("runtime projection group members must be unique")
            expected_start = 0
            for member in self.members:
                if member.row_start != expected_start:
                    raise ValueError("runtime projection group slices must be contiguous")
                expected_start = member.row_end
            if expected_start != self.out_features:
                raise ValueError("runtime projection group slices must cover the output")


@dataclass(frozen=True, slots=True)
class WorkloadSpec:
    """Shape of the calls a plan will make (reference ``backend.py:76-91``)."""

    kind: WorkloadKind
    device_type: str
    input_dtype: str
    batch_size: int
    token_count: int
    deterministic: bool = False

    def __post_init__(self) -> None:
        if self.kind not in ("prefill", "decode"):
            raise ValueError(f"unsupported runtime workload kind: {self.kind}")
        if not self.device_type:
            raise ValueError("runtime workload device type must be non-empty")
        if self.batch_size <= 0 or self.token_count <= 0:
            raise ValueError("runtime workload batch and token counts must be positive")


@dataclass(frozen=True, slots=True)
class BackendCapabilities:
    """Static capability declaration (reference ``backend.py:94-122``)."""

    logical_formats: tuple[str, ...]
    device_types: tuple[str, ...]
    input_dtypes: tuple[str, ...]
    factor_dtypes: tuple[str, ...]
    scale_dtypes: tuple[str, ...]
    outlier_value_dtypes: tuple[str, ...]
    workload_kinds: tuple[WorkloadKind, ...]
    supports_bias: bool
    supports_outliers: bool
    supports_deterministic: bool
    in_feature_alignment: int = 1
    out_feature_alignment: int = 1
    rank_alignment: int = 1
    maximum_batch_size: int | None = None
    maximum_token_count: int | None = None
    patch_value_dtypes: tuple[str, ...] = ()

    def __post_init__(self) -> None:
        if not (self.logical_formats and self.device_types and self.input_dtypes):
            raise ValueError("runtime backend capabilities must declare formats, devices, and input dtypes")
        if min(self.in_feature_alignment, self.out_feature_alignment, self.rank_alignment) < 1:
            raise ValueError("runtime backend alignments must be positive")
        if self.maximum_batch_size is not None and self.maximum_batch_size < 1:
            raise ValueError("runtime backend maximum batch size must be positive")
        if self.maximum_token_count is not None and self.maximum_token_count < 1:
            raise ValueError("runtime backend maximum token count must be positive")


@dataclass(frozen=True, slots=True)
class SupportResult:
    """Outcome of ``supports`` with a stable code (reference ``backend.py:125-138``)."""

    supported: bool
    code: str
    reason: str

    @classmethod
    def accepted(cls) -> SupportResult:
        return cls(True, "NQ-INF-OK", "supported")

    @classmethod
    def rejected(cls, code: str, reason: str) -> SupportResult:
        if not (code and reason):
            raise ValueError("runtime backend rejection requires a code and reason")
        return cls(False, code, reason)


@runtime_checkable
class RuntimeLayerState(Protocol):
    @property
    def spec(self) -> QuantizedLinearSpec: ...


@dataclass(frozen=True, slots=True)
class PreparedLayer:
    """Device-resident payload produced by ``prepare`` (reference ``backend.py:147-152``)."""

    backend_name: str
    backend_version: str
    spec: QuantizedLinearSpec
    payload: object


@runtime_checkable
class RuntimeBackend(Protocol):
    """The four-call operator protocol (reference ``backend.py:155-166``)."""

    name: str
    version: str

    def capabilities(self) -> BackendCapabilities: ...

    def supports(self, op: QuantizedLinearSpec, workload: WorkloadSpec) -> SupportResult: ...

    def prepare(self, state: RuntimeLayerState, device: DeviceLike) -> PreparedLayer: ...

    def linear(self, value: torch.Tensor, layer: PreparedLayer) -> torch.Tensor: ...


def evaluate_capabilities(
    capabilities: BackendCapabilities,
    op: QuantizedLinearSpec,
    workload: WorkloadSpec,
) -> SupportResult:
    """Return the first failing capability check, in the reference's order.

    The order and codes follow ``backend.py:169-266`` of the reference exactly,
    because planners report the first code and callers match on it.
    """

    caps = capabilities
    ordered_checks = [
        ("NQ-INF-FORMAT", lambda: op.logical_format in caps.logical_formats,
         lambda: f"logical format {op.logical_format!r} is not supported"),
        ("NQ-INF-DEVICE", lambda: workload.device_type in caps.device_types,
         lambda: f"device type {workload.device_type!r} is not supported"),
        ("NQ-INF-INPUT-DTYPE", lambda: workload.input_dtype in caps.input_dtypes,
         lambda: f"input dtype {workload.input_dtype!r} is not supported"),
        ("NQ-INF-FACTOR-DTYPE", lambda: op.factor_dtype in caps.factor_dtypes,
         lambda: f"factor dtype {op.factor_dtype!r} is not supported"),
        ("NQ-INF-SCALE-DTYPE", lambda: op.scale_dtype in caps.scale_dtypes,
         lambda: f"scale dtype {op.scale_dtype!r} is not supported"),
        ("NQ-INF-WORKLOAD", lambda: workload.kind in caps.workload_kinds,
         lambda: f"workload kind {workload.kind!r} is not supported"),
        ("NQ-INF-BIAS", lambda: (not op.has_bias) or caps.supports_bias,
         lambda: "bias is not supported"),
        ("NQ-INF-BIAS-DTYPE", lambda: op.bias_dtype is None or op.bias_dtype in caps.scale_dtypes,
         lambda: f"bias dtype {op.bias_dtype!r} is not supported"),
        ("NQ-INF-OUTLIERS", lambda: op.outlier_count == 0 or caps.supports_outliers,
         lambda: "salient outliers are not supported"),
        ("NQ-INF-OUTLIER-DTYPE",
         lambda: op.outlier_value_dtype is None or op.outlier_value_dtype in caps.outlier_value_dtypes,
         lambda: f"outlier dtype {op.outlier_value_dtype!r} is not supported"),
        ("NQ-INF-PATCH",
         lambda: op.patch_value_dtype is None or op.patch_value_dtype in caps.patch_value_dtypes,
         lambda: f"low-rank patch dtype {op.patch_value_dtype!r} is not supported"),
        ("NQ-INF-DETERMINISM", lambda: (not workload.deterministic) or caps.supports_deterministic,
         lambda: "deterministic execution is not supported"),
        ("NQ-INF-IN-ALIGNMENT", lambda: op.in_features % caps.in_feature_alignment == 0,
         lambda: f"input features must be aligned to {caps.in_feature_alignment}"),
        ("NQ-INF-OUT-ALIGNMENT", lambda: op.out_features % caps.out_feature_alignment == 0,
         lambda: f"output features must be aligned to {caps.out_feature_alignment}"),
        ("NQ-INF-RANK-ALIGNMENT", lambda: op.rank % caps.rank_alignment == 0,
         lambda: f"rank must be aligned to {caps.rank_alignment}"),
        ("NQ-INF-BATCH",
         lambda: caps.maximum_batch_size is None or workload.batch_size <= caps.maximum_batch_size,
         lambda: f"batch size {workload.batch_size} exceeds the backend maximum"),
        ("NQ-INF-TOKENS",
         lambda: caps.maximum_token_count is None or workload.token_count <= caps.maximum_token_count,
         lambda: f"token count {workload.token_count} exceeds the backend maximum"),
    ]
    for code, passes, reason in ordered_checks:
        if not passes():
            return SupportResult.rejected(code, reason())
    return SupportResult.accepted()


__all__ = [
    "BackendCapabilities",
    "DeviceLike",
    "PreparedLayer",
    "ProjectionMemberSpec",
    "QuantizedLinearSpec",
    "RuntimeBackend",
    "RuntimeLayerState",
    "SupportResult",
    "WorkloadKind",
    "WorkloadSpec",
    "evaluate_capabilities",
]
