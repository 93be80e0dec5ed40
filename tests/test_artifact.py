"""Packed model artifacts: the reference's on-disk format (``nanoquant_b200.artifact``).

``tests/golden/packed_artifact`` was written by the reference's own writer
(``tests/golden/make_golden.py``), and ``packed_artifact_layers.npz`` holds
what the reference's ``load_layer`` returned for each layer.  CPU tests check
that this package reads the same tensors and rejects the same corruptions;
the ``gpu`` test loads the artifact straight onto the device with the batched
value checks, prepares it and runs it against the oracle.
"""

from __future__ import annotations

import json
import shutil

import numpy as np
import pytest
import torch

from nanoquant_b200.artifact import PackedArtifactError, open_packed_artifact
from tests.fixtures import GOLDEN, load

ROOT = GOLDEN / "packed_artifact"
FIELDS = ("left_words", "right_words", "scale_pre", "scale_mid", "scale_post", "bias", "outlier_indices",
          "outlier_values", "outlier_scales", "patch_left", "patch_right")


def _copy(tmp_path):
    target = tmp_path / "artifact"
    shutil.copytree(ROOT, target)
    return target


def test_layers_match_the_reference_loader() -> None:
    artifact = open_packed_artifact(ROOT)
    expected = load("packed_artifact_layers")
    names = artifact.layer_names()
    assert names == ("blocks.0.self_attn.q_proj", "blocks.0.mlp.up_proj", "blocks.1.self_attn.o_proj")
    for name in names:
        state = artifact.load_layer(name)
        for field in FIELDS:
            value = getattr(state, field)
            key = f"{name}:{field}"
            if key not in expected:
                assert value is None, key
                continue
            assert value is not None and value.dtype == expected[key].dtype, key
            assert torch.equal(value, expected[key]), key


def test_open_checks_headers_without_loading(tmp_path) -> None:
    artifact = open_packed_artifact(ROOT)
    assert artifact.manifest.layer_count == 3 and len(artifact.manifest.blocks) == 2
    with pytest.raises(KeyError):
        artifact.load_layer("blocks.9.missing")


def test_rejects_a_corrupt_shard(tmp_path) -> None:
    root = _copy(tmp_path)
    shard = root / "weights" / "block-00000.safetensors"
    data = bytearray(shard.read_bytes())
    data[-1] ^= 0x01
    shard.write_bytes(bytes(data))
    with pytest.raises(PackedArtifactError, match="hash"):
        open_packed_artifact(root)


def test_rejects_future_schema_and_noncanonical_keys(tmp_path) -> None:
    root = _copy(tmp_path)
    descriptor = root / "nanoquant-packed-model.json"
    payload = json.loads(descriptor.read_text())
    payload["schema_version"] = 2
    descriptor.write_text(json.dumps(payload))
    with pytest.raises(PackedArtifactError, match="schema"):
        open_packed_artifact(root)
    payload["schema_version"] = 1
    payload["blocks"][0]["layers"][0]["tensors"][0]["key"] = "other.key"
    descriptor.write_text(json.dumps(payload))
    with pytest.raises(PackedArtifactError, match="key"):
        open_packed_artifact(root)


def test_rejects_a_path_outside_the_root(tmp_path) -> None:
    root = _copy(tmp_path)
    descriptor = root / "nanoquant-packed-model.json"
    payload = json.loads(descriptor.read_text())
    payload["blocks"][0]["path"] = "../block.safetensors"
    descriptor.write_text(json.dumps(payload))
    with pytest.raises(PackedArtifactError, match="canonical"):
        open_packed_artifact(root)


def _flip_padding_bit(root) -> None:
    """Set a padding bit of the first layer's right words in place (the hash check is skipped)."""

    from safetensors.torch import load_file, save_file

    shard = root / "weights" / "block-00000.safetensors"
    tensors = load_file(shard)
    key = "layouts.llama.cpp-i32-lsb-v1.blocks.0.self_attn.q_proj.factor_right_words"
    tensors[key][0, -1] |= 1 << 30  # 35 columns: bits 3..31 of the last word are padding
    size = shard.stat().st_size
    save_file(tensors, shard)
    assert shard.stat().st_size == size


def test_value_checks_are_the_constructor_checks(tmp_path) -> None:
    root = _copy(tmp_path)
    _flip_padding_bit(root)
    artifact = open_packed_artifact(root, verify_hashes=False)
    with pytest.raises(ValueError, match="padding"):
        artifact.load_layer("blocks.0.self_attn.q_proj")


class _CpuBackend:
    def prepare(self, state, device):  # noqa: ARG002
        return state


def test_deferred_block_checks_raise_the_first_failure(tmp_path) -> None:
    root = _copy(tmp_path)
    _flip_padding_bit(root)
    artifact = open_packed_artifact(root, verify_hashes=False)
    with pytest.raises(ValueError, match="padding"):
        artifact.prepare_block(0, _CpuBackend(), "cpu")
    states = artifact.prepare_block(1, _CpuBackend(), "cpu")
    assert list(states) == ["blocks.1.self_attn.o_proj"]


@pytest.mark.gpu
def test_device_load_prepare_and_run_match_the_oracle(tmp_path) -> None:
    if not torch.cuda.is_available():
        pytest.fail("GPU test needs CUDA")
    from nanoquant_b200 import CudaPackedSm100Backend
    from oracle import packed_oracle as po
    from tests.test_cuda_parity import oracle_from_state

    backend = CudaPackedSm100Backend()
    artifact = open_packed_artifact(ROOT)
    prepared = artifact.prepare_all(backend, "cuda")
    g = torch.Generator().manual_seed(3)
    for name, layer in prepared.items():
        state = artifact.load_layer(name)
        x = torch.randn(4, state.spec.in_features, generator=g).bfloat16()
        got = backend.linear(x.cuda(), layer).cpu()
        expected = po.packed_linear(x.float().numpy(), oracle_from_state(state), accumulate="float64")
        np.testing.assert_allclose(got.numpy(), expected, rtol=2e-5, atol=2e-4 * max(1.0, np.abs(expected).max()))
    # a corrupted padding bit is caught by the batched device checks
    root = _copy(tmp_path)
    _flip_padding_bit(root)
    with pytest.raises(ValueError, match="padding"):
        open_packed_artifact(root, verify_hashes=False).prepare_block(0, backend, "cuda")
