"""Packed model artifacts: the reference's on-disk format, loaded onto the GPU.

Reads the block-sharded artifact the reference writes
(``src/nanoquant/runtime/packed_artifact.py:306-420``): a directory holding
``nanoquant-packed-model.json`` (the manifest: schema, layout, model metadata,
blocks of layers with their specs and tensor inventories) and one safetensors
shard per block under ``weights/``.  ``open_packed_artifact`` checks the
manifest, shard sizes and hashes and every tensor header without reading
payloads, and ``load_layer`` returns a ``PackedLayerState`` like the
reference's (same names, same errors).

``prepare_block`` is the load path of the CUDA backend: it reads one shard's
tensors straight to the device, builds the block's layers with their value
checks (padding bits, finiteness, salient-column invariants) evaluated on the
device and copied back in one transfer instead of one host synchronisation per
check, and prepares them with the given backend.
"""

from __future__ import annotations

import hashlib
import json
from dataclasses import dataclass
from pathlib import Path, PurePosixPath
from typing import Any

import torch

from nanoquant_b200.backend import DeviceLike, PreparedLayer, ProjectionMemberSpec, QuantizedLinearSpec
from nanoquant_b200.packed import (
    PACKED_LAYOUT_VERSION,
    PACKED_TENSOR_NAMESPACE,
    PACKED_WORD_BITS,
    PACKED_WORD_DTYPE,
    PackedLayerState,
    deferred_value_checks,
    packed_word_count,
)

PACKED_ARTIFACT_FORMAT = "nanoquant-packed-model"
PACKED_ARTIFACT_DESCRIPTOR = "nanoquant-packed-model.json"
PACKED_DESCRIPTOR_SCHEMA_VERSION = 1  # reference constants.py:12
MINIMUM_RUNTIME_VERSION = "0.1.0"  # reference artifact.py:23
_MAXIMUM_DESCRIPTOR_BYTES = 16 * 1024 * 1024
_SAFETENSORS_DTYPES = {"F16": "float16", "BF16": "bfloat16", "F32": "float32", "I8": "int8", "I16": "int16",
                       "I32": "int32", "I64": "int64", "U8": "uint8"}
_ROLES = ("factor_left_words", "factor_right_words", "scale_pre", "scale_mid", "scale_post", "bias",
          "outlier_indices", "outlier_values", "outlier_scales", "patch_left", "patch_right")


class PackedArtifactError(ValueError):
    """A packed artifact is missing, malformed or inconsistent (reference packed_artifact.py:58-59)."""


@dataclass(frozen=True, slots=True)
class PackedTensorEntry:
    role: str
    key: str
    shape: tuple[int, ...]
    dtype: str


@dataclass(frozen=True, slots=True)
class PackedLayerEntry:
    spec: QuantizedLinearSpec
    tensors: tuple[PackedTensorEntry, ...]


@dataclass(frozen=True, slots=True)
class PackedBlockEntry:
    index: int
    path: str
    bytes: int
    sha256: str
    layers: tuple[PackedLayerEntry, ...]


@dataclass(frozen=True, slots=True)
class PackedModelManifest:
    schema_version: int
    artifact_format: str
    minimum_runtime_version: str
    layout: dict[str, Any]
    model: dict[str, str]
    logical_descriptor_sha256: str
    blocks: tuple[PackedBlockEntry, ...]
    layer_count: int
    weight_bytes: int


def _expected_tensors(spec: QuantizedLinearSpec) -> dict[str, tuple[tuple[int, ...], str]]:
    """Role -> (shape, dtype) a layer of ``spec`` stores (reference packed_artifact.py:80-114)."""

    out: dict[str, tuple[tuple[int, ...], str]] = {
        "factor_left_words": ((spec.out_features, packed_word_count(spec.rank)), "int32"),
        "factor_right_words": ((spec.rank, packed_word_count(spec.in_features)), "int32"),
        "scale_pre": ((spec.in_features,), spec.scale_dtype),
        "scale_mid": ((spec.rank,), spec.scale_dtype),
        "scale_post": ((spec.out_features,), spec.scale_dtype),
    }
    if spec.has_bias:
        out["bias"] = ((spec.out_features,), spec.bias_dtype or spec.scale_dtype)
    if spec.outlier_count:
        out["outlier_indices"] = ((spec.outlier_count,), "int32")
        out["outlier_values"] = ((spec.out_features, spec.outlier_count), str(spec.outlier_value_dtype))
    if spec.has_outlier_scales:
        out["outlier_scales"] = ((spec.outlier_count,), spec.scale_dtype)
    if spec.patch_rank:
        out["patch_left"] = ((spec.out_features, spec.patch_rank), str(spec.patch_value_dtype))
        out["patch_right"] = ((spec.patch_rank, spec.in_features), str(spec.patch_value_dtype))
    return out


def _relative_path(value: str) -> None:
    path = PurePosixPath(value)
    if (not value or "\\" in value or path.is_absolute() or any(part in ("", ".", "..") for part in path.parts)
            or path.as_posix() != value):
        raise PackedArtifactError(f"packed artifact path is not canonical and relative: {value!r}")


def _member(root: Path, relative: str) -> Path:
    _relative_path(relative)
    resolved = (root / relative).resolve()
    if root.resolve() not in resolved.parents:
        raise PackedArtifactError(f"packed artifact member escapes its root: {relative}")
    return resolved


def _sha256(path: Path) -> str:
    digest = hashlib.sha256()
    with path.open("rb") as stream:
        for chunk in iter(lambda: stream.read(1 << 20), b""):
            digest.update(chunk)
    return digest.hexdigest()


def _is_digest(value: object) -> bool:
    return isinstance(value, str) and len(value) == 64 and all(c in "0123456789abcdef" for c in value)


def _spec(payload: dict[str, Any]) -> QuantizedLinearSpec:
    fields = dict(payload)
    fields["members"] = tuple(ProjectionMemberSpec(**member) for member in fields.get("members", ()))
    return QuantizedLinearSpec(**fields)


def _layer(payload: dict[str, Any]) -> PackedLayerEntry:
    spec = _spec(payload["spec"])
    tensors = tuple(PackedTensorEntry(t["role"], t["key"], tuple(int(d) for d in t["shape"]), t["dtype"])
                    for t in payload["tensors"])
    by_role = {tensor.role: tensor for tensor in tensors}
    if len(by_role) != len(tensors):
        raise PackedArtifactError(f"packed layer tensor roles are duplicated: {spec.name}")
    if any(role not in _ROLES for role in by_role):
        raise PackedArtifactError(f"unsupported packed tensor role in layer {spec.name}")
    expected = _expected_tensors(spec)
    if set(by_role) != set(expected):
        raise PackedArtifactError(f"packed layer tensor inventory differs from its specification: {spec.name}")
    for role, (shape, dtype) in expected.items():
        tensor = by_role[role]
        if tensor.key != f"{PACKED_TENSOR_NAMESPACE}.{spec.name}.{role}":
            raise PackedArtifactError(f"packed layer tensor key differs: {spec.name}:{role}")
        if tensor.shape != shape or tensor.dtype != dtype:
            raise PackedArtifactError(f"packed layer tensor metadata differs: {spec.name}:{role}")
    return PackedLayerEntry(spec, tensors)


def _manifest(payload: dict[str, Any]) -> PackedModelManifest:
    """Decode and check the manifest (reference packed_artifact.py:159-189)."""

    if payload.get("schema_version") != PACKED_DESCRIPTOR_SCHEMA_VERSION:
        raise PackedArtifactError(f"unsupported packed artifact schema: {payload.get('schema_version')}")
    if payload.get("artifact_format") != PACKED_ARTIFACT_FORMAT:
        raise PackedArtifactError(f"unsupported packed artifact format: {payload.get('artifact_format')}")
    if payload.get("minimum_runtime_version") != MINIMUM_RUNTIME_VERSION:
        raise PackedArtifactError(
            f"unsupported packed minimum runtime version: {payload.get('minimum_runtime_version')}")
    layout = dict(payload["layout"])
    if (layout.get("version"), layout.get("word_dtype"), layout.get("word_bits")) != (
            PACKED_LAYOUT_VERSION, PACKED_WORD_DTYPE, PACKED_WORD_BITS):
        raise PackedArtifactError("packed artifact layout differs from layout v1")
    if (layout.get("bit_order"), layout.get("positive_bit"), layout.get("negative_bit"),
            layout.get("padding_bit")) != ("least-significant-bit-first", 0, 1, 0):
        raise PackedArtifactError("packed artifact sign encoding differs from layout v1")
    if layout.get("tensor_namespace") != PACKED_TENSOR_NAMESPACE:
        raise PackedArtifactError("packed artifact tensor namespace differs from layout v1")
    model = dict(payload["model"])
    if not all(model.get(k) for k in ("source", "revision", "family", "config_hash", "tokenizer_hash")):
        raise PackedArtifactError("runtime model metadata fields must be non-empty")
    if not _is_digest(payload.get("logical_descriptor_sha256")):
        raise PackedArtifactError("packed source descriptor hash must be lowercase SHA-256")
    blocks = []
    for block in payload["blocks"]:
        layers = tuple(_layer(layer) for layer in block["layers"])
        entry = PackedBlockEntry(int(block["index"]), block["path"], int(block["bytes"]), block["sha256"], layers)
        if entry.bytes <= 0 or not _is_digest(entry.sha256):
            raise PackedArtifactError(f"packed block {entry.index} size or hash is invalid")
        _relative_path(entry.path)
        names = [layer.spec.name for layer in layers]
        if not names or len(names) != len(set(names)):
            raise PackedArtifactError("packed block must contain uniquely named layers")
        blocks.append(entry)
    if not blocks or [b.index for b in blocks] != list(range(len(blocks))):
        raise PackedArtifactError(f"packed artifact blocks are not contiguous: {[b.index for b in blocks]}")
    names = [layer.spec.name for block in blocks for layer in block.layers]
    if len(names) != len(set(names)) or len(names) != payload["layer_count"]:
        raise PackedArtifactError("packed artifact layer count or uniqueness is inconsistent")
    if sum(block.bytes for block in blocks) != payload["weight_bytes"]:
        raise PackedArtifactError("packed artifact weight byte count is inconsistent")
    return PackedModelManifest(payload["schema_version"], payload["artifact_format"],
                               payload["minimum_runtime_version"], layout, model,
                               payload["logical_descriptor_sha256"], tuple(blocks), len(names),
                               payload["weight_bytes"])


def _state(entry: PackedLayerEntry, loaded: dict[str, torch.Tensor]) -> PackedLayerState:
    by_role = {tensor.role: loaded[tensor.key] for tensor in entry.tensors}
    return PackedLayerState(
        entry.spec, PACKED_LAYOUT_VERSION, by_role["factor_left_words"], by_role["factor_right_words"],
        by_role["scale_pre"], by_role["scale_mid"], by_role["scale_post"], by_role.get("bias"),
        by_role.get("outlier_indices"), by_role.get("outlier_values"), by_role.get("outlier_scales"),
        by_role.get("patch_left"), by_role.get("patch_right"))


def _read(path: Path, keys: list[str], device: DeviceLike) -> dict[str, torch.Tensor]:
    from safetensors import safe_open

    target = torch.device(device)
    out: dict[str, torch.Tensor] = {}
    with safe_open(path, framework="pt", device="cpu") as handle:
        available = set(handle.keys())
        missing = [key for key in keys if key not in available]
        if missing:
            raise KeyError(f"safetensors keys are missing: {tuple(missing)}")
        for key in keys:
            value = handle.get_tensor(key)
            out[key] = value if target.type == "cpu" else value.to(target, non_blocking=True)
    return out


@dataclass(frozen=True, slots=True)
class OpenPackedArtifact:
    """An opened artifact (reference packed_artifact.py:191-224)."""

    root: Path
    manifest: PackedModelManifest

    def _find(self, name: str) -> tuple[PackedBlockEntry, PackedLayerEntry]:
        matches = [(block, layer) for block in self.manifest.blocks for layer in block.layers
                   if layer.spec.name == name]
        if len(matches) != 1:
            raise KeyError(f"packed artifact layer not found: {name}")
        return matches[0]

    def layer_names(self) -> tuple[str, ...]:
        return tuple(layer.spec.name for block in self.manifest.blocks for layer in block.layers)

    def load_layer(self, name: str, device: DeviceLike = "cpu") -> PackedLayerState:
        """One validated packed layer on ``device`` (the reference's ``load_layer``)."""

        block, layer = self._find(name)
        loaded = _read(self.root / block.path, [tensor.key for tensor in layer.tensors], device)
        return _state(layer, loaded)

    def prepare_block(self, index: int, backend, device: DeviceLike) -> dict[str, PreparedLayer]:
        """Read block ``index`` onto ``device``, validate it with one device round trip, prepare every layer.

        Raises the ``ValueError`` of the first failed check, in layer order;
        nothing of the block is returned then.
        """

        block = self.manifest.blocks[index]
        keys = [tensor.key for layer in block.layers for tensor in layer.tensors]
        loaded = _read(self.root / block.path, keys, device)
        with deferred_value_checks():
            states = [_state(layer, loaded) for layer in block.layers]
        return {state.spec.name: backend.prepare(state, device) for state in states}

    def prepare_all(self, backend, device: DeviceLike) -> dict[str, PreparedLayer]:
        """``prepare_block`` over every block, in order."""

        out: dict[str, PreparedLayer] = {}
        for index in range(len(self.manifest.blocks)):
            out.update(self.prepare_block(index, backend, device))
        return out


def open_packed_artifact(root: str | Path, *, verify_hashes: bool = True) -> OpenPackedArtifact:
    """Check the manifest, shard sizes, hashes and tensor headers without loading payloads
    (reference packed_artifact.py:379-420)."""

    from safetensors import safe_open

    artifact_root = Path(root)
    descriptor = artifact_root / PACKED_ARTIFACT_DESCRIPTOR
    if not descriptor.is_file():
        raise PackedArtifactError("packed artifact descriptor is missing")
    if descriptor.stat().st_size > _MAXIMUM_DESCRIPTOR_BYTES:
        raise PackedArtifactError("packed artifact descriptor exceeds the size limit")
    try:
        manifest = _manifest(json.loads(descriptor.read_text(encoding="utf-8")))
    except PackedArtifactError:
        raise
    except (OSError, UnicodeError, json.JSONDecodeError, KeyError, TypeError, ValueError) as error:
        raise PackedArtifactError(f"packed artifact descriptor is invalid: {error}") from error
    for block in manifest.blocks:
        shard = _member(artifact_root, block.path)
        if not shard.is_file() or shard.stat().st_size != block.bytes:
            raise PackedArtifactError(f"packed artifact shard size or presence differs: {block.path}")
        if verify_hashes and _sha256(shard) != block.sha256:
            raise PackedArtifactError(f"packed artifact shard hash differs: {block.path}")
        declared = {tensor.key: tensor for layer in block.layers for tensor in layer.tensors}
        if len(declared) != sum(len(layer.tensors) for layer in block.layers):
            raise PackedArtifactError(f"packed artifact tensor key is duplicated: {block.path}")
        try:
            with safe_open(shard, framework="pt", device="cpu") as handle:
                if set(handle.keys()) != set(declared):
                    raise PackedArtifactError(f"packed artifact shard tensor inventory differs: {block.path}")
                for key, tensor in declared.items():
                    view = handle.get_slice(key)
                    dtype = _SAFETENSORS_DTYPES.get(str(view.get_dtype()))
                    if tuple(view.get_shape()) != tensor.shape or dtype != tensor.dtype:
                        raise PackedArtifactError(f"packed artifact tensor header differs: {block.path}:{key}")
        except PackedArtifactError:
            raise
        except Exception as error:
            raise PackedArtifactError(f"packed artifact shard header is invalid: {block.path}") from error
    return OpenPackedArtifact(artifact_root.resolve(), manifest)


__all__ = [
    "MINIMUM_RUNTIME_VERSION",
    "OpenPackedArtifact",
    "PACKED_ARTIFACT_DESCRIPTOR",
    "PACKED_ARTIFACT_FORMAT",
    "PACKED_DESCRIPTOR_SCHEMA_VERSION",
    "PackedArtifactError",
    "PackedBlockEntry",
    "PackedLayerEntry",
    "PackedModelManifest",
    "PackedTensorEntry",
    "open_packed_artifact",
]
