"""Host-side format code of ``nanoquant_b200`` against the reference's fixtures (CPU)."""

from __future__ import annotations

from dataclasses import replace

import numpy as np
import pytest
import torch

from nanoquant_b200 import (
    PACKED_LAYOUT_VERSION,
    LogicalLayerState,
    PackedLayerState,
    PackedLayoutMetadata,
    QuantizedLinearSpec,
    pack_logical_layer,
    pack_product_codebook_indices,
    pack_product_half_table,
    pack_sign_matrix,
    packed_row_stride_bytes,
    packed_word_count,
    supports_vector_word_loads,
    unpack_product_codebook_indices,
    unpack_product_half_table,
    unpack_sign_matrix,
)
from nanoquant_b200.product_codebook import ProductCodebookLayerState, decode_product_codebook_right_words
from tests.fixtures import load


@pytest.mark.parametrize("columns", (1, 31, 32, 33, 65, 128))
def test_pack_sign_matrix_matches_reference_words(columns: int) -> None:
    fixture = load("packing")
    signs = torch.from_numpy(fixture[f"signs_{columns}"])
    words = pack_sign_matrix(signs)
    assert words.dtype == torch.int32
    assert words.shape == (3, packed_word_count(columns))
    assert np.array_equal(words.numpy(), fixture[f"words_{columns}"])
    assert torch.equal(unpack_sign_matrix(words, 3, columns), signs)


def test_bit_order_known_answer() -> None:
    values = torch.ones(2, 32)
    values[0, (0, 1, 31)] = -1
    values[1] = -1
    packed = pack_sign_matrix(values)
    assert int(packed[0, 0]) == -(2**31) + 3
    assert int(packed[1, 0]) == -1


def test_unpack_rejects_noncanonical_padding() -> None:
    packed = pack_sign_matrix(torch.ones(1, 33))
    packed[0, -1] = 2
    with pytest.raises(ValueError, match="non-zero padding bit"):
        unpack_sign_matrix(packed, 1, 33)


def test_row_stride_controls_vector_loads() -> None:
    assert packed_row_stride_bytes(33) == 8
    assert packed_row_stride_bytes(128) == 16
    assert not supports_vector_word_loads(pack_sign_matrix(torch.ones(2, 33)))
    assert supports_vector_word_loads(pack_sign_matrix(torch.ones(2, 128)))


def test_pack_rejects_non_signs() -> None:
    with pytest.raises(ValueError, match="other than -1 or"):
        pack_sign_matrix(torch.tensor([[1.0, 0.0]]))


def _logical(factor_dtype: torch.dtype = torch.float32) -> LogicalLayerState:
    spec = QuantizedLinearSpec(
        "blocks.0.linear", "nanoquant-v1", 35, 3, 33, str(factor_dtype).removeprefix("torch."), "float32",
        outlier_count=2, outlier_value_dtype="int8", has_outlier_scales=True, has_bias=True,
    )
    left = torch.where(torch.arange(99).reshape(3, 33) % 2 == 0, 1.0, -1.0).to(factor_dtype)
    right = torch.where(torch.arange(33 * 35).reshape(33, 35) % 5 == 0, -1.0, 1.0).to(factor_dtype)
    return LogicalLayerState(
        spec, left, right,
        torch.cat((torch.tensor([0.5, 0.0]), torch.linspace(0.5, 1.5, 32), torch.zeros(1))),
        torch.linspace(0.75, 1.25, 33), torch.linspace(1.0, 1.5, 3), torch.tensor([0.1, -0.2, 0.3]),
        torch.tensor([1, 34], dtype=torch.int32), torch.tensor([[1, -2], [3, -4], [5, -6]], dtype=torch.int8),
        torch.tensor([0.25, 0.5]),
    )


@pytest.mark.parametrize("factor_dtype", (torch.float16, torch.bfloat16, torch.float32))
def test_packed_layer_roundtrip(factor_dtype: torch.dtype) -> None:
    logical = _logical(factor_dtype)
    packed = pack_logical_layer(logical)
    restored = packed.to_logical()
    assert packed.layout == PACKED_LAYOUT_VERSION
    assert packed.left_words.shape == (3, 2) and packed.right_words.shape == (33, 2)
    for expected, actual in (
        (logical.left_binary, restored.left_binary),
        (logical.right_binary, restored.right_binary),
        (logical.scale_pre, restored.scale_pre),
        (logical.outlier_values, restored.outlier_values),
    ):
        assert torch.equal(expected, actual)


def test_packed_layer_rejects_nonzero_pre_at_salient_columns() -> None:
    logical = _logical()
    pre = logical.scale_pre.clone()
    pre[logical.outlier_indices.long()] = 1
    with pytest.raises(ValueError, match="exactly zero scale_pre"):
        PackedLayerState(
            logical.spec, PACKED_LAYOUT_VERSION, pack_sign_matrix(logical.left_binary),
            pack_sign_matrix(logical.right_binary), pre, logical.scale_mid, logical.scale_post, logical.bias,
            logical.outlier_indices, logical.outlier_values, logical.outlier_scales,
        )


def test_packed_layer_rejects_scales_for_float_outliers() -> None:
    packed = pack_logical_layer(_logical())
    with pytest.raises(ValueError, match="scales require int8"):
        PackedLayerState(
            replace(packed.spec, outlier_value_dtype="float32"), packed.layout, packed.left_words,
            packed.right_words, packed.scale_pre, packed.scale_mid, packed.scale_post, packed.bias,
            packed.outlier_indices, packed.outlier_values.float(), packed.outlier_scales,
        )


def test_layout_metadata() -> None:
    layout = PackedLayoutMetadata()
    assert layout.version == "llama.cpp-i32-lsb-v1"
    assert (layout.positive_bit, layout.negative_bit, layout.padding_bit) == (0, 1, 0)


def test_spec_validation_messages() -> None:
    with pytest.raises(ValueError, match="canonical dotted path"):
        QuantizedLinearSpec("/bad", "nanoquant-v1", 4, 3, 2, "float32", "float32")
    with pytest.raises(ValueError, match="must be positive"):
        QuantizedLinearSpec("a.b", "nanoquant-v1", 0, 3, 2, "float32", "float32")
    with pytest.raises(ValueError, match="outlier dtype must be present"):
        QuantizedLinearSpec("a.b", "nanoquant-v1", 4, 3, 2, "float32", "float32", outlier_count=1)


def test_product_codebook_stream_known_answer() -> None:
    fixture = load("product_codebook")
    indices = torch.from_numpy(fixture["kat_indices"])
    payload = pack_product_codebook_indices(indices)
    assert payload.shape == (8,)
    assert np.array_equal(payload.numpy(), fixture["kat_payload"])
    assert torch.equal(unpack_product_codebook_indices(payload, (3, 5)), indices)
    payload[-1] |= torch.tensor(1 << 16, dtype=torch.int32)
    with pytest.raises(ValueError, match="non-zero padding"):
        unpack_product_codebook_indices(payload, (3, 5))


def _codebook_state(fixture: dict, tag: str) -> ProductCodebookLayerState:
    n, m, r, free_rows, transposed = (int(v) for v in fixture[f"{tag}_shape"])
    spec = QuantizedLinearSpec(f"blocks.0.{tag}", "nanoquant-v1", n, m, r, "float32", "float16")
    return ProductCodebookLayerState(
        spec, "product-codebook-free-k16-v1", bool(transposed), free_rows,
        fixture[f"{tag}_factor_left_words"], fixture[f"{tag}_factor_right_free_words"],
        fixture[f"{tag}_factor_right_coded_payload"], fixture[f"{tag}_first_half_words"],
        fixture[f"{tag}_second_half_words"], fixture[f"{tag}_factor_scale_pre"],
        fixture[f"{tag}_factor_scale_mid"], fixture[f"{tag}_factor_scale_post"],
    )


@pytest.mark.parametrize("tag", ("small", "small_t", "c4like"))
def test_product_codebook_to_packed_matches_reference(tag: str) -> None:
    fixture = load("product_codebook")
    state = _codebook_state(fixture, tag)
    packed = state.to_packed()
    assert torch.equal(packed.right_words, fixture[f"{tag}_right_words"])
    assert torch.equal(packed.left_words, fixture[f"{tag}_left_words"])
    assert torch.equal(packed.scale_pre, fixture[f"{tag}_scale_pre"])


def test_product_half_table_roundtrip() -> None:
    g = torch.Generator().manual_seed(3)
    table = torch.where(torch.rand(256, 16, generator=g) > 0.5, 1.0, -1.0)
    words = pack_product_half_table(table)
    assert words.dtype == torch.int16 and words.shape == (256,)
    assert torch.equal(unpack_product_half_table(words), table)


def test_decode_product_codebook_matches_reference() -> None:
    fixture = load("product_codebook")
    n, m, r, free_rows, _ = (int(v) for v in fixture["c4like_shape"])
    words = decode_product_codebook_right_words(
        fixture["c4like_factor_right_free_words"], fixture["c4like_factor_right_coded_payload"],
        fixture["c4like_first_half_words"], fixture["c4like_second_half_words"], rank=r, columns=n,
    )
    assert torch.equal(words, fixture["c4like_right_words"])
