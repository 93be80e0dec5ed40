"""B200 (sm_100a) runtime backend for the packed binary low-rank linear.

:class:`CudaPackedSm100Backend` implements the four-call ``RuntimeBackend``
protocol of the reference runtime (``src/nanoquant/runtime/backend.py:155-166``)
and is a drop-in for ``CudaPackedBackend``
(``src/nanoquant/runtime/cuda_backend.py:151-278``): same capability table,
same ``prepare``/``linear`` contract and error types, fp32 output on the
current stream.  All arithmetic runs in ``libnqb.so`` through its C ABI; there
is no Python or library fallback, and every entry point raises when the
library or a CUDA device is missing.

The grouped-projection helpers mirror ``prepare_cuda_projection_group`` and
``grouped_cuda_projection`` (reference ``cuda_backend.py:65-144``).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, fields

import torch

from nanoquant_b200 import _native
from nanoquant_b200.backend import (
    BackendCapabilities,
    DeviceLike,
    PreparedLayer,
    ProjectionMemberSpec,
    QuantizedLinearSpec,
    RuntimeLayerState,
    SupportResult,
    WorkloadSpec,
    evaluate_capabilities,
)
from nanoquant_b200.logical import canonical_torch_dtype
from nanoquant_b200.overlay import OutlierRowOverlay, OverlaidLayerState
from nanoquant_b200.packed import PACKED_LAYOUT_VERSION, PackedLayerState
from nanoquant_b200.mixed_v import MixedVLayerState
from nanoquant_b200.product_codebook import ProductCodebookLayerState

CUDA_SM100_BACKEND_NAME = "cuda-packed-sm100a"
CUDA_SM100_BACKEND_VERSION = "1"
_FLOAT_DTYPES = ("float16", "bfloat16", "float32")


@dataclass(frozen=True, slots=True)
class _Sm100Payload:
    """Device tensors of one prepared layer; ``desc`` points into them."""

    device: torch.device
    tensors: dict[str, torch.Tensor]
    desc: _native.LinearDesc
    patch_left: torch.Tensor | None
    patch_right: torch.Tensor | None


def _to_device(value: torch.Tensor | None, device: torch.device) -> torch.Tensor | None:
    return None if value is None else value.detach().to(device=device).contiguous()


def _repack(words: torch.Tensor, rows: int, columns: int) -> torch.Tensor:
    """Kernel-native tile copy of a layout-v1 sign matrix (``nqb_repack_signs``)."""

    size = ctypes.c_size_t(0)
    _native.call("nqb_repack_bytes", rows, columns, ctypes.byref(size))
    tiles = torch.empty(size.value, dtype=torch.uint8, device=words.device)
    _native.call("nqb_repack_signs", words.data_ptr(), rows, columns, tiles.data_ptr(),
                 _native.current_stream_handle(words.device))
    return tiles


# A grouped call runs on the tensor-core paths while its members' 128-row
# tiles (rank and output rows) fit the library's 4096 completion counters;
# layers up to a third of that stay eligible in any group of three.
_TILES_ONLY_MAX_ROW_TILES = 4096 // 3


def _build_payload(
    state: PackedLayerState | ProductCodebookLayerState | MixedVLayerState,
    overlay: OutlierRowOverlay | None,
    device: torch.device,
    tensor_cores: bool = True,
    coded_mixed_v: bool = False,
    coded_product_codebook: bool = True,
    keep_words: bool = False,
) -> _Sm100Payload:
    spec = state.spec
    tensors: dict[str, torch.Tensor] = {}

    def keep(name: str, value: torch.Tensor | None) -> torch.Tensor | None:
        moved = _to_device(value, device)
        if moved is not None:
            tensors[name] = moved
        return moved

    desc = _native.LinearDesc()
    desc.in_features = spec.in_features
    desc.out_features = spec.out_features
    desc.rank = spec.rank
    patch_left = patch_right = None
    if isinstance(state, ProductCodebookLayerState) and not state.factorization_transposed:
        # canonical orientation: keep V compact, the kernels decode records in flight
        desc.left_words = keep("left_words", state.factor_left_words).data_ptr()
        desc.codebook_free_rows = state.free_rows
        desc.codebook_free_words = keep("codebook_free_words", state.factor_right_free_words).data_ptr()
        desc.codebook_payload = keep("codebook_payload", state.factor_right_coded_payload).data_ptr()
        desc.codebook_first = keep("codebook_first", state.first_half_words).data_ptr()
        desc.codebook_second = keep("codebook_second", state.second_half_words).data_ptr()
        scale_pre, scale_mid, scale_post = state.factor_scale_pre, state.factor_scale_mid, state.factor_scale_post
        outliers = (state.outlier_indices, state.outlier_values, state.outlier_scales)
        bias = None
        if tensor_cores:
            # the tensor-core paths read kernel-native tiles: decode V on the
            # device once and tile both factors (the compact records stay the
            # generic kernels' input)
            from nanoquant_b200.device_ops import decode_product_codebook_cuda

            right_words = decode_product_codebook_cuda(
                tensors["codebook_free_words"], tensors["codebook_payload"], tensors["codebook_first"],
                tensors["codebook_second"], rank=spec.rank, columns=spec.in_features)
            tensors["left_tiles"] = _repack(tensors["left_words"], spec.out_features, spec.rank)
            tensors["right_tiles"] = _repack(right_words, spec.rank, spec.in_features)
            desc.left_tiles = tensors["left_tiles"].data_ptr()
            desc.right_tiles = tensors["right_tiles"].data_ptr()
            if coded_product_codebook:
                # decode programs stream V's coded rows as 16-bit records and
                # decode them through the two half-word tables in stage 1
                from nanoquant_b200.device_ops import repack_product_codebook_cuda

                tensors["coded_right_tiles"], tensors["coded_codebook"] = repack_product_codebook_cuda(
                    tensors["codebook_payload"].contiguous(), tensors["codebook_first"].contiguous(),
                    tensors["codebook_second"].contiguous(), rank=spec.rank, columns=spec.in_features,
                    free_rows=state.free_rows)
                desc.coded_right_tiles = tensors["coded_right_tiles"].data_ptr()
                desc.coded_codebook = tensors["coded_codebook"].data_ptr()
                desc.coded_free_rows = state.free_rows
                desc.coded_format = _native.NQB_CODED_PRODUCT_CODEBOOK
    else:
        if isinstance(state, MixedVLayerState):
            # expand the 19-bit records once on the device, like the reference
            # backend (cuda_backend.py:209-224); the layer then runs as packed
            from nanoquant_b200.device_ops import decode_mixed_v_cuda

            tensors["right_words"] = decode_mixed_v_cuda(
                _to_device(state.free_right_words, device), _to_device(state.coded_payload, device),
                _to_device(state.codebook_words, device), rank=spec.rank, columns=spec.in_features)
            packed = state
        else:
            packed = state.to_packed() if isinstance(state, ProductCodebookLayerState) else state
            keep("right_words", packed.right_words)
        desc.left_words = keep("left_words", packed.left_words).data_ptr()
        desc.right_words = tensors["right_words"].data_ptr()
        scale_pre, scale_mid, scale_post = packed.scale_pre, packed.scale_mid, packed.scale_post
        outliers = (packed.outlier_indices, packed.outlier_values, packed.outlier_scales)
        bias = packed.bias
        patch_left = keep("patch_left", packed.patch_left)
        patch_right = keep("patch_right", packed.patch_right)
        if tensor_cores:
            tensors["left_tiles"] = _repack(tensors["left_words"], spec.out_features, spec.rank)
            tensors["right_tiles"] = _repack(tensors["right_words"], spec.rank, spec.in_features)
            desc.left_tiles = tensors["left_tiles"].data_ptr()
            desc.right_tiles = tensors["right_tiles"].data_ptr()
            if coded_mixed_v and isinstance(state, MixedVLayerState):
                # decode programs stream V's coded rows as records and decode them in stage 1
                from nanoquant_b200.device_ops import repack_mixed_v_cuda

                codebook = tensors.setdefault("coded_codebook",
                                              _to_device(state.codebook_words, device).contiguous().clone())
                tensors["coded_right_tiles"] = repack_mixed_v_cuda(
                    _to_device(state.coded_payload, device).contiguous(), rank=spec.rank, columns=spec.in_features,
                    free_rows=state.free_rows)
                desc.coded_right_tiles = tensors["coded_right_tiles"].data_ptr()
                desc.coded_codebook = codebook.data_ptr()
                desc.coded_free_rows = state.free_rows
                desc.coded_format = _native.NQB_CODED_MIXED_V
    desc.scale_pre = keep("scale_pre", scale_pre).data_ptr()
    desc.scale_mid = keep("scale_mid", scale_mid).data_ptr()
    desc.scale_post = keep("scale_post", scale_post).data_ptr()
    desc.scale_dtype = _native.dtype_code(scale_pre.dtype)
    if bias is not None:
        desc.bias = keep("bias", bias).data_ptr()
        desc.bias_dtype = _native.dtype_code(bias.dtype)
    indices, values, scales = outliers
    if indices is not None and values is not None:
        desc.outlier_count = int(indices.numel())
        desc.outlier_indices = keep("outlier_indices", indices.to(torch.int32)).data_ptr()
        desc.outlier_values = keep("outlier_values", values).data_ptr()
        desc.outlier_value_dtype = _native.dtype_code(values.dtype)
        if scales is not None:
            desc.outlier_scales = keep("outlier_scales", scales.reshape(-1)).data_ptr()
    if overlay is not None:
        desc.overlay_rows = int(overlay.row_ids.numel())
        desc.overlay_row_ids = keep("overlay_row_ids", overlay.row_ids).data_ptr()
        desc.overlay_values = keep("overlay_values", overlay.values).data_ptr()
        desc.overlay_scales = keep("overlay_scales", overlay.scales).data_ptr()
        desc.overlay_scale_dtype = _native.dtype_code(overlay.scales.dtype)
    if patch_left is not None and patch_right is not None:
        # the library applies the patch inside nqb_linear (fused into the decode stages)
        desc.patch_rank = int(patch_left.shape[1])
        desc.patch_left = patch_left.data_ptr()
        desc.patch_right = patch_right.data_ptr()
        desc.patch_dtype = _native.dtype_code(patch_left.dtype)
    row_tiles = -(-spec.rank // 128) + -(-spec.out_features // 128)
    if tensor_cores and not keep_words and row_tiles <= _TILES_ONLY_MAX_ROW_TILES:
        # tiles-only layer: every call shape it can take runs on the tensor-core
        # decode, prefill or program paths, which read the tiles only, so the
        # layout-v1 words (and a codebook layer's compact V) leave the device
        for name in ("left_words", "right_words", "codebook_free_words", "codebook_payload", "codebook_first",
                     "codebook_second"):
            tensors.pop(name, None)
        desc.left_words = desc.right_words = None
        desc.codebook_free_words = desc.codebook_payload = desc.codebook_first = desc.codebook_second = None
    return _Sm100Payload(device, tensors, desc, patch_left, patch_right)


def _adopt_spec(spec) -> QuantizedLinearSpec:
    """This package's spec with the fields of ``spec`` (an instance of the reference's equal dataclass)."""

    if isinstance(spec, QuantizedLinearSpec):
        return spec
    values = {f.name: getattr(spec, f.name) for f in fields(QuantizedLinearSpec)}
    values["members"] = tuple(ProjectionMemberSpec(m.name, m.row_start, m.row_end) for m in values["members"])
    return QuantizedLinearSpec(**values)


_ADOPTABLE = {cls.__name__: cls for cls in (PackedLayerState, MixedVLayerState, ProductCodebookLayerState)}


def adopt_layer_state(state: object) -> object:
    """The reference runtime's own layer states as this package's equal types.

    The reference loader (``packed_artifact.py:196-223``) and planner
    (``planning.py:234-260``) hand ``prepare`` instances of
    ``nanoquant.runtime``'s ``PackedLayerState``, ``MixedVLayerState`` and
    ``ProductCodebookLayerState``; their fields are the ones this package's
    classes declare (same names, meanings and tensor layouts), so such a state
    is rebuilt field by field, through this package's validation.  Other
    objects are returned unchanged.
    """

    target = _ADOPTABLE.get(type(state).__name__)
    if target is None or isinstance(state, target):
        return state
    try:
        values = {f.name: getattr(state, f.name) for f in fields(target)}
    except AttributeError as error:
        raise TypeError(f"{type(state).__module__}.{type(state).__name__} lacks a field of {target.__name__}: "
                        f"{error}") from error
    values["spec"] = _adopt_spec(values["spec"])
    return target(**values)


def _cuda_device(device: DeviceLike) -> torch.device:
    target = torch.device(device)
    if target.type != "cuda":
        raise ValueError("sm100a packed backend preparation requires a CUDA device")
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is not available in this runtime")
    if target.index is None:
        target = torch.device("cuda", torch.cuda.current_device())
    return target


def _check_input(value: torch.Tensor, spec: QuantizedLinearSpec, device: torch.device) -> None:
    """The input contract of the reference ``CudaPackedBackend.linear`` (cuda_backend.py:249-262)."""

    if value.device != device:
        raise ValueError("CUDA packed input and prepared layer must use the same device")
    if canonical_torch_dtype(value.dtype) not in _FLOAT_DTYPES:
        raise ValueError(f"CUDA packed input dtype is unsupported: {value.dtype}")
    if value.ndim == 0 or value.shape[-1] != spec.in_features:
        raise ValueError("CUDA packed input feature dimension differs from the layer")
    if value.numel() == 0:
        raise ValueError("CUDA packed input must contain at least one token")
    if not value.is_contiguous():
        raise ValueError("CUDA packed input must be contiguous")
    if value.requires_grad:
        raise ValueError("CUDA packed runtime does not support autograd")


def _workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


# One zero-initialised libnqb workspace per (device, stream): calls on a stream
# are ordered, and every call leaves the workspace's counter region zero, so
# the buffer is reused across layers and calls (like a per-stream BLAS
# workspace).  It only grows; a grown buffer starts zeroed again.
_STREAM_WORKSPACES: dict[tuple[int, int], torch.Tensor] = {}


def stream_workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    key = (device.index if device.index is not None else torch.cuda.current_device(),
           torch.cuda.current_stream(device).cuda_stream)
    current = _STREAM_WORKSPACES.get(key)
    if current is None or current.numel() < nbytes:
        # (during CUDA-graph capture the zero fill becomes a node of the graph)
        current = torch.zeros(max(int(nbytes), 1 << 16), dtype=torch.uint8, device=device)
        _STREAM_WORKSPACES[key] = current
    return current


def kernel_path(layer: PreparedLayer, tokens: int, input_dtype: torch.dtype = torch.bfloat16) -> str:
    """Which kernels ``linear`` runs for ``tokens`` tokens: ``"tensor-core"``, ``"prefill"`` or ``"generic"``."""

    if not isinstance(layer.payload, _Sm100Payload):
        raise TypeError("prepared runtime layer has an invalid sm100a packed payload")
    path = ctypes.c_int32(-1)
    _native.call("nqb_linear_path", ctypes.byref(layer.payload.desc), 1, _native.dtype_code(input_dtype), tokens,
                 ctypes.byref(path))
    return {_native.NQB_PATH_TENSOR_CORE: "tensor-core", _native.NQB_PATH_PREFILL: "prefill"}.get(path.value, "generic")


def packed_linear(value: torch.Tensor, payload: _Sm100Payload, spec: QuantizedLinearSpec,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """Run one prepared layer on ``value`` (any leading shape) and return fp32 ``[..., out]``.

    ``out``, when given, is a contiguous fp32 tensor of ``tokens * out_features``
    elements on the same device that receives the result (no allocation).
    """

    tokens = value.numel() // spec.in_features
    if out is None:
        output = torch.empty((*value.shape[:-1], spec.out_features), dtype=torch.float32, device=value.device)
    else:
        if (out.dtype != torch.float32 or not out.is_contiguous() or out.device != value.device
                or out.numel() != tokens * spec.out_features):
            raise ValueError("out must be a contiguous fp32 tensor of tokens * out_features elements on x's device")
        output = out
    needed = ctypes.c_size_t(0)
    desc_ref = ctypes.byref(payload.desc)
    _native.call("nqb_linear_workspace_bytes", desc_ref, tokens, ctypes.byref(needed))
    workspace = stream_workspace(needed.value, value.device)
    stream = _native.current_stream_handle(value.device)
    _native.call(
        "nqb_linear",
        desc_ref,
        value.data_ptr(),
        _native.dtype_code(value.dtype),
        tokens,
        output.data_ptr(),
        workspace.data_ptr(),
        workspace.numel(),
        stream,
    )
    return output


class CudaPackedSm100Backend:
    """sm_100a two-stage packed linear behind the reference ``RuntimeBackend`` protocol."""

    name = CUDA_SM100_BACKEND_NAME
    version = CUDA_SM100_BACKEND_VERSION
    packed_layout = PACKED_LAYOUT_VERSION

    def __init__(self, *, tensor_cores: bool = True, coded_mixed_v: bool = False,
                 coded_product_codebook: bool = True, keep_words: bool = False) -> None:
        # tensor_cores=False keeps prepared layers on the CUDA-core kernels only
        # (no kernel-native tile copies); used to cross-check the two paths.
        # coded_mixed_v=True also keeps a mixed-V layer's V as coded tiles, which
        # decode programs stream and decode in stage 1 (38 % fewer V bytes; at
        # batch 1 the record decode costs more time than the bytes save, so the
        # expanded tiles are the default).
        # coded_product_codebook (the default) does the same for a
        # product-codebook layer's V: 16-bit records, half the bytes of sign
        # words, decoded through the two half-word tables in the program's
        # stage 1 (within 1 % of the expanded tiles' time at batch 1 and 16,
        # where the step is latency-bound).  The per-call paths keep
        # streaming the expanded tiles.
        self.tensor_cores = tensor_cores
        self.coded_mixed_v = coded_mixed_v
        self.coded_product_codebook = coded_product_codebook
        # keep_words=True keeps the layout-v1 words on the device after the
        # tile copies are made; without it a tensor-core layer holds its
        # tiles only (half the sign memory), and a call that would take the
        # generic path (more than 2^22 tokens) raises.
        self.keep_words = keep_words

    def capabilities(self) -> BackendCapabilities:
        return BackendCapabilities(
            logical_formats=("nanoquant-v1",),
            device_types=("cuda",),
            input_dtypes=_FLOAT_DTYPES,
            factor_dtypes=_FLOAT_DTYPES,
            scale_dtypes=_FLOAT_DTYPES,
            outlier_value_dtypes=(*_FLOAT_DTYPES, "int8"),
            workload_kinds=("prefill", "decode"),
            supports_bias=True,
            supports_outliers=True,
            supports_deterministic=True,
            patch_value_dtypes=_FLOAT_DTYPES,
        )

    def supports(self, op: QuantizedLinearSpec, workload: WorkloadSpec) -> SupportResult:
        result = evaluate_capabilities(self.capabilities(), op, workload)
        if not result.supported:
            return result
        try:
            _native.library()
        except (RuntimeError, OSError) as error:
            return SupportResult.rejected("NQ-INF-CUDA-KERNEL", str(error))
        if not torch.cuda.is_available():
            return SupportResult.rejected("NQ-INF-DEVICE-UNAVAILABLE", "CUDA is not available in this runtime")
        capability = torch.cuda.get_device_capability()
        if capability != (10, 0):
            return SupportResult.rejected(
                "NQ-INF-CUDA-CAPABILITY",
                f"CUDA compute capability {capability[0]}.{capability[1]} is not sm_100 (B200)",
            )
        return result

    def prepare(self, state: RuntimeLayerState, device: DeviceLike) -> PreparedLayer:
        """Copy ``state`` to ``device`` and build the kernel-native tiles.

        Accepts this package's layer states and the reference runtime's own
        (adopted field by field, :func:`adopt_layer_state`); the returned
        layer carries ``state.spec`` itself, so the reference planner's
        ``layer.spec == state.spec`` check holds (``planning.py:251-253``).
        """

        overlay = None
        base = adopt_layer_state(state)
        if isinstance(base, OverlaidLayerState):
            base, overlay = adopt_layer_state(base.base), base.overlay
        if not isinstance(base, (PackedLayerState, ProductCodebookLayerState, MixedVLayerState)):
            raise TypeError(
                "sm100a packed backend requires PackedLayerState, MixedVLayerState, "
                "ProductCodebookLayerState or OverlaidLayerState"
            )
        target = _cuda_device(device)
        _native.library()
        with torch.cuda.device(target):
            payload = _build_payload(base, overlay, target, self.tensor_cores, self.coded_mixed_v,
                                     self.coded_product_codebook, self.keep_words)
        return PreparedLayer(self.name, self.version, state.spec, payload)

    def linear(self, value: torch.Tensor, layer: PreparedLayer) -> torch.Tensor:
        if layer.backend_name != self.name or layer.backend_version != self.version:
            raise ValueError("prepared runtime layer belongs to a different backend")
        if not isinstance(layer.payload, _Sm100Payload):
            raise TypeError("prepared runtime layer has an invalid sm100a packed payload")
        _check_input(value, layer.spec, layer.payload.device)
        return packed_linear(value, layer.payload, layer.spec)

    def linear_into(self, value: torch.Tensor, layer: PreparedLayer, out: torch.Tensor) -> torch.Tensor:
        """:meth:`linear` writing into ``out`` (contiguous fp32, ``tokens * out_features`` elements)."""

        if layer.backend_name != self.name or layer.backend_version != self.version:
            raise ValueError("prepared runtime layer belongs to a different backend")
        if not isinstance(layer.payload, _Sm100Payload):
            raise TypeError("prepared runtime layer has an invalid sm100a packed payload")
        _check_input(value, layer.spec, layer.payload.device)
        return packed_linear(value, layer.payload, layer.spec, out)


@dataclass(frozen=True, slots=True)
class Sm100ProjectionGroup:
    """Two or three prepared layers sharing one input, run as one grouped call."""

    device: torch.device
    layers: tuple[PreparedLayer, ...]
    descs: ctypes.Array  # type: ignore[type-arg]
    in_features: int
    output_features: tuple[int, ...]


def prepare_sm100_projection_group(layers: tuple[PreparedLayer, ...]) -> Sm100ProjectionGroup | None:
    """Group compatible prepared layers (reference ``prepare_cuda_projection_group``, cuda_backend.py:65-120).

    Returns ``None`` when the layers cannot share one call, as the reference does.
    Unlike the reference, ranks and widths need no 8-alignment and bias,
    int8 outlier scales, overlays and a low-rank patch are allowed (the
    library applies each member's patch inside the grouped call).
    """

    if len(layers) not in (2, 3):
        return None
    payloads = tuple(layer.payload for layer in layers)
    if not all(isinstance(payload, _Sm100Payload) for payload in payloads):
        return None
    first = payloads[0]
    in_features = layers[0].spec.in_features
    if any(payload.device != first.device for payload in payloads):
        return None
    if any(layer.spec.in_features != in_features for layer in layers):
        return None
    if any(payload.desc.scale_dtype != first.desc.scale_dtype for payload in payloads):
        return None
    descs = (_native.LinearDesc * len(layers))(*(payload.desc for payload in payloads))
    return Sm100ProjectionGroup(
        first.device,
        tuple(layers),
        descs,
        in_features,
        tuple(layer.spec.out_features for layer in layers),
    )


def grouped_sm100_projection(value: torch.Tensor, group: Sm100ProjectionGroup) -> tuple[torch.Tensor, ...]:
    """Run a projection group on ``value``; returns one fp32 tensor per member."""

    if value.device != group.device:
        raise ValueError("grouped CUDA projection input uses a different device")
    _check_input(value, group.layers[0].spec, group.device)
    tokens = value.numel() // group.in_features
    outputs = tuple(
        torch.empty((*value.shape[:-1], width), dtype=torch.float32, device=value.device)
        for width in group.output_features
    )
    count = len(group.layers)
    needed = ctypes.c_size_t(0)
    _native.call("nqb_grouped_workspace_bytes", group.descs, count, tokens, ctypes.byref(needed))
    workspace = stream_workspace(needed.value, value.device)
    out_ptrs = (ctypes.c_void_p * count)(*(out.data_ptr() for out in outputs))
    _native.call(
        "nqb_grouped_linear",
        group.descs,
        count,
        value.data_ptr(),
        _native.dtype_code(value.dtype),
        tokens,
        out_ptrs,
        workspace.data_ptr(),
        workspace.numel(),
        _native.current_stream_handle(value.device),
    )
    return outputs


# Names of the reference module, for callers that import them directly.
prepare_cuda_projection_group = prepare_sm100_projection_group
grouped_cuda_projection = grouped_sm100_projection


__all__ = [
    "CUDA_SM100_BACKEND_NAME",
    "CUDA_SM100_BACKEND_VERSION",
    "CudaPackedSm100Backend",
    "Sm100ProjectionGroup",
    "adopt_layer_state",
    "grouped_cuda_projection",
    "grouped_sm100_projection",
    "kernel_path",
    "packed_linear",
    "prepare_cuda_projection_group",
    "prepare_sm100_projection_group",
]
