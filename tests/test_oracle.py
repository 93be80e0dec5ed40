"""Pin the CPU oracle against the reference's own outputs (golden fixtures).

These run on CPU.  Integer/bit work must match bit-exactly; the fp32 linear
must match the reference's fp32 result within fp32 rounding noise.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import packed_oracle as po
from tests.fixtures import as_numpy_f32, linear_names, load


def oracle_layer(case: dict) -> po.OracleLayer:
    def get(name):
        value = case.get(name)
        if value is None:
            return None
        if hasattr(value, "numpy"):
            if name in ("left_words", "right_words", "outlier_indices") or str(value.dtype) == "torch.int8":
                return value.numpy()
            return as_numpy_f32(value)
        return value

    return po.OracleLayer(
        int(case["in_features"]), int(case["out_features"]), int(case["rank"]),
        get("left_words"), get("right_words"), get("scale_pre"), get("scale_mid"), get("scale_post"),
        get("bias"), get("outlier_indices"), get("outlier_values"), get("outlier_scales"),
        get("patch_left"), get("patch_right"),
    )


def test_bit_order_known_answer() -> None:
    # bits (0, 1, 31) set -> -(2**31) + 3 and all bits set -> -1
    # (reference tests/unit/test_runtime_packed.py:62-70)
    signs = np.ones((2, 32), dtype=np.float32)
    signs[0, (0, 1, 31)] = -1
    signs[1] = -1
    words = po.pack_signs(signs)
    assert int(words[0, 0]) == -(2**31) + 3
    assert int(words[1, 0]) == -1
    fixture = load("packing")
    assert np.array_equal(words, fixture["kat_words"])


@pytest.mark.parametrize("columns", (1, 31, 32, 33, 65, 128))
def test_pack_matches_reference_words(columns: int) -> None:
    fixture = load("packing")
    for prefix in ("", "pattern_"):
        signs = fixture[f"signs_{columns}" if not prefix else f"pattern_{columns}"]
        expected = fixture[f"words_{columns}" if not prefix else f"pattern_words_{columns}"]
        words = po.pack_signs(signs)
        assert words.dtype == np.int32
        assert np.array_equal(words, expected)
        assert np.array_equal(po.unpack_signs(words, 3, columns), signs)


def test_pack_large_matrix_matches_reference() -> None:
    fixture = load("packing")
    assert np.array_equal(po.pack_signs(fixture["big_signs"]), fixture["big_words"])


def test_unpack_rejects_nonzero_padding() -> None:
    words = po.pack_signs(np.ones((1, 33), dtype=np.float32))
    words[0, -1] = 2
    with pytest.raises(ValueError, match="non-zero padding bit"):
        po.unpack_signs(words, 1, 33)


@pytest.mark.parametrize("name", linear_names())
def test_oracle_linear_matches_reference(name: str) -> None:
    case = load(name)
    layer = oracle_layer(case)
    x = as_numpy_f32(case["x"])
    expected = case["y"].numpy()
    actual = po.packed_linear(x, layer)
    assert actual.shape == expected.shape
    # both sides are fp32 sgemm results; only summation order differs
    np.testing.assert_allclose(actual, expected, rtol=1e-5, atol=1e-5 * max(1.0, float(np.abs(expected).max())))


@pytest.mark.parametrize("index", (0, 1, 2))
def test_oracle_grouped_members_match_reference(index: int) -> None:
    case = load(f"grouped_{index}")
    layer = oracle_layer(case)
    actual = po.packed_linear(case["x"].numpy(), layer)
    expected = case["y"].numpy()
    np.testing.assert_allclose(actual, expected, rtol=1e-5, atol=1e-6 * float(np.abs(expected).max()))


def test_product_codebook_record_stream_known_answer() -> None:
    fixture = load("product_codebook")
    # 15 records -> 8 words (reference tests/unit/test_runtime_product_codebook.py:63-72)
    assert fixture["kat_payload"].shape == (8,)
    records = po.unpack_codebook_records(fixture["kat_payload"], 15)
    assert np.array_equal(records.reshape(3, 5).astype(np.int32), fixture["kat_indices"])
    padded = fixture["kat_payload"].copy()
    padded[-1] |= np.int32(1 << 16)
    with pytest.raises(ValueError, match="non-zero padding"):
        po.unpack_codebook_records(padded, 15)


@pytest.mark.parametrize("tag", ("small", "c4like"))
def test_product_codebook_decode_matches_reference(tag: str) -> None:
    fixture = load("product_codebook")
    n, m, r, free_rows, transposed = (int(v) for v in fixture[f"{tag}_shape"])
    assert not transposed
    words = po.decode_codebook_right_words(
        fixture[f"{tag}_factor_right_free_words"].numpy(),
        fixture[f"{tag}_factor_right_coded_payload"].numpy(),
        fixture[f"{tag}_first_half_words"].numpy(),
        fixture[f"{tag}_second_half_words"].numpy(),
        r,
        n,
    )
    assert np.array_equal(words, fixture[f"{tag}_right_words"].numpy())
    layer = po.OracleLayer(
        n, m, r, fixture[f"{tag}_left_words"].numpy(), words,
        as_numpy_f32(fixture[f"{tag}_scale_pre"]), as_numpy_f32(fixture[f"{tag}_factor_scale_mid"]),
        as_numpy_f32(fixture[f"{tag}_scale_post"]),
    )
    actual = po.packed_linear(as_numpy_f32(fixture[f"{tag}_x"]), layer)
    np.testing.assert_allclose(actual, fixture[f"{tag}_y"].numpy(), rtol=1e-5, atol=1e-6)


def test_mixed_v_record_stream_known_answer() -> None:
    fixture = load("mixed_v")
    # 34 records of 19 bits -> 21 words (reference tests/unit/test_runtime_mixed_v.py:32-44)
    assert fixture["kat_payload"].shape == (21,)
    index, pair = po.unpack_mixed_v_records(fixture["kat_payload"], 34)
    assert np.array_equal(index.reshape(2, 17), fixture["kat_indices"])
    assert np.array_equal(pair.reshape(2, 17), fixture["kat_pairs"])
    decoded = po.decode_mixed_v_right_words(fixture["free"], fixture["payload"], fixture["codebook"], 7, 64)
    assert np.array_equal(decoded, fixture["decoded"])


def test_row_overlay_definition() -> None:
    # the overlay has no reference type: check the definition on a hand example
    rng = np.random.default_rng(0)
    words_u = po.pack_signs(np.where(rng.random((4, 3)) > 0.5, 1.0, -1.0))
    words_v = po.pack_signs(np.where(rng.random((3, 5)) > 0.5, 1.0, -1.0))
    layer = po.OracleLayer(5, 4, 3, words_u, words_v, np.ones(5, np.float32), np.ones(3, np.float32),
                           np.ones(4, np.float32))
    x = rng.standard_normal((2, 5)).astype(np.float32)
    base = po.packed_linear(x, layer)
    layer.overlay_row_ids = np.array([1, 3], dtype=np.int32)
    layer.overlay_values = np.array([[1, -2, 3, 0, 5], [-1, 0, 0, 2, 0]], dtype=np.int8)
    layer.overlay_scales = np.array([0.5, 0.25], dtype=np.float32)
    with_overlay = po.packed_linear(x, layer)
    delta = with_overlay - base
    np.testing.assert_allclose(delta[:, 0], 0)
    np.testing.assert_allclose(delta[:, 1], 0.5 * (x @ layer.overlay_values[0].astype(np.float32)), rtol=1e-6)
    np.testing.assert_allclose(delta[:, 3], 0.25 * (x @ layer.overlay_values[1].astype(np.float32)), rtol=1e-6)
