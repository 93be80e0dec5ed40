"""Mixed-V right factor (``mixed-v-free-k10-pair9-v1``): host container, oracle and device decode.

CPU tests pin the host restatement (``nanoquant_b200.mixed_v``) to the
reference's golden record stream and to the oracle; the ``gpu`` tests check
the device decode (``nqb_decode_mixed_v``) bit for bit and run mixed-V layers
through every kernel path of the backend against the oracle.
"""

from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch

from nanoquant_b200 import (
    LogicalLayerState,
    MixedVLayerState,
    QuantizedLinearSpec,
    decode_mixed_v_right_words,
    mixed_v_correction_pair_table,
    mixed_v_from_packed_words,
    mixed_v_payload_word_count,
    pack_logical_layer,
    pack_mixed_v_records,
    packed_word_count,
    unpack_mixed_v_records,
)
from oracle import packed_oracle as po
from tests.fixtures import load


def _pair_flips() -> np.ndarray:
    table = mixed_v_correction_pair_table().numpy()[:496].astype(np.int64)
    return ((1 << (table & 0xFF)) | (1 << ((table >> 8) & 0xFF))).astype(np.uint32)


def _records(n: int, coded_rows: int, rng: np.random.Generator) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Codebook and records whose decoded words keep the padding bits of a ragged last word zero.

    Records of the last word of a row use codebook entries 960..1023, each
    stored pre-flipped by its own pair so that the decode clears the flip.
    """

    wpr = packed_word_count(n)
    book = rng.integers(0, 2**32, 1024, dtype=np.uint64).astype(np.uint32)
    index = rng.integers(0, 960, (coded_rows, wpr)).astype(np.int32)
    pair = rng.integers(0, 496, (coded_rows, wpr)).astype(np.int32)
    tail = n % 32
    if tail:
        own_pair = rng.integers(0, 496, 64).astype(np.int32)
        low = rng.integers(0, 2**32, 64, dtype=np.uint64).astype(np.uint32) & np.uint32((1 << tail) - 1)
        book[960:] = low ^ _pair_flips()[own_pair]
        entry = rng.integers(0, 64, coded_rows)
        index[:, -1] = 960 + entry
        pair[:, -1] = own_pair[entry]
    return book.view(np.int32), index, pair


def mixed_v_state(n: int, m: int, r: int, free_rows: int, seed: int, *, bias: bool = False,
                  outliers: int = 0) -> MixedVLayerState:
    """Random mixed-V layer: random U, free V rows and records; fp16 scales |N(0,1)| * 0.05 + 0.01."""

    g = torch.Generator().manual_seed(seed)
    rng = np.random.default_rng(seed)
    spec = QuantizedLinearSpec(
        "blocks.0.mlp.up_proj", "nanoquant-v1", n, m, r, "float32", "float16",
        outlier_count=outliers, outlier_value_dtype="int8" if outliers else None,
        has_outlier_scales=bool(outliers), has_bias=bias,
    )
    pre = (torch.randn(n, generator=g).abs() * 0.05 + 0.01).half()
    idx = None
    if outliers:
        idx = torch.sort(torch.randperm(n, generator=g)[:outliers]).values
        pre[idx] = 0
    packed = pack_logical_layer(LogicalLayerState(
        spec,
        torch.where(torch.rand(m, r, generator=g) > 0.5, 1.0, -1.0),
        torch.where(torch.rand(r, n, generator=g) > 0.5, 1.0, -1.0),
        pre,
        (torch.randn(r, generator=g).abs() + 0.5).half(),
        (torch.randn(m, generator=g).abs() * 0.05 + 0.01).half(),
        bias=torch.randn(m, generator=g).half() if bias else None,
        outlier_indices=idx,
        outlier_values=torch.randint(-127, 128, (m, outliers), generator=g, dtype=torch.int8) if outliers else None,
        outlier_scales=torch.full((outliers,), 0.002).half() if outliers else None,
    ))
    book, index, pair = _records(n, r - free_rows, rng)
    coded = book.view(np.uint32)[index] ^ _pair_flips()[pair]
    right = torch.cat((packed.right_words[:free_rows], torch.from_numpy(coded.view(np.int32))), dim=0).contiguous()
    packed = dataclasses.replace(packed, right_words=right)
    return mixed_v_from_packed_words(packed, free_rows=free_rows, codebook_words=torch.from_numpy(book),
                                     codebook_indices=torch.from_numpy(index),
                                     correction_pair_ids=torch.from_numpy(pair))


# ------------------------------------------------------------------ CPU ---


def test_record_stream_matches_reference_known_answer() -> None:
    fixture = load("mixed_v")
    payload = pack_mixed_v_records(torch.from_numpy(fixture["kat_indices"]), torch.from_numpy(fixture["kat_pairs"]))
    assert payload.shape == (21,) and np.array_equal(payload.numpy(), fixture["kat_payload"])
    index, pair = unpack_mixed_v_records(payload, (2, 17))
    assert np.array_equal(index.numpy(), fixture["kat_indices"])
    assert np.array_equal(pair.numpy(), fixture["kat_pairs"])
    words = decode_mixed_v_right_words(torch.from_numpy(fixture["free"]), torch.from_numpy(fixture["payload"]),
                                       torch.from_numpy(fixture["codebook"]), rank=7, in_features=64)
    assert np.array_equal(words.numpy(), fixture["decoded"])


def test_pair_table_enumerates_every_pair_once() -> None:
    table = mixed_v_correction_pair_table().numpy()
    assert table.shape == (512,) and not table[496:].any()
    pairs = [(int(v) & 0xFF, int(v) >> 8) for v in table[:496]]
    assert pairs == sorted(pairs) and len(set(pairs)) == 496
    assert all(a < b < 32 for a, b in pairs)


@pytest.mark.parametrize("count", (1, 27, 32, 33, 1000))
def test_random_streams_round_trip_and_match_the_oracle(count: int) -> None:
    rng = np.random.default_rng(count)
    index = torch.from_numpy(rng.integers(0, 1024, (1, count)).astype(np.int32))
    pair = torch.from_numpy(rng.integers(0, 496, (1, count)).astype(np.int32))
    payload = pack_mixed_v_records(index, pair)
    assert payload.numel() == mixed_v_payload_word_count(count)
    got_index, got_pair = unpack_mixed_v_records(payload, (1, count))
    assert torch.equal(got_index, index) and torch.equal(got_pair, pair)
    o_index, o_pair = po.unpack_mixed_v_records(payload.numpy(), count)
    assert np.array_equal(o_index.reshape(1, count), index.numpy())
    assert np.array_equal(o_pair.reshape(1, count), pair.numpy())


@pytest.mark.parametrize(("n", "r", "free_rows"), ((64, 7, 2), (97, 40, 1), (640, 480, 17), (1152, 209, 100)))
def test_state_decode_matches_oracle(n: int, r: int, free_rows: int) -> None:
    state = mixed_v_state(n, 96, r, free_rows, seed=n + r)
    words = state.to_packed().right_words
    oracle = po.decode_mixed_v_right_words(state.free_right_words.numpy(), state.coded_payload.numpy(),
                                           state.codebook_words.numpy(), r, n)
    assert np.array_equal(words.numpy(), oracle)
    assert state.record_count == (r - free_rows) * packed_word_count(n)


def test_state_validation_errors() -> None:
    state = mixed_v_state(64, 32, 8, 2, seed=1)
    with pytest.raises(ValueError, match="format"):
        dataclasses.replace(state, format="mixed-v-other")
    with pytest.raises(ValueError, match="free row"):
        dataclasses.replace(state, free_rows=8)
    with pytest.raises(ValueError, match="1024"):
        dataclasses.replace(state, codebook_words=state.codebook_words[:512].contiguous())
    bad_padding = state.coded_payload.clone()
    bad_padding[-1] |= torch.tensor(-(2**31), dtype=torch.int32)  # top bit of the stream, past the last record
    with pytest.raises(ValueError, match="padding"):
        dataclasses.replace(state, coded_payload=bad_padding)
    # a record naming pair id 500 (valid 10-bit index, invalid pair)
    index = torch.zeros((1, 1), dtype=torch.int32)
    payload = pack_mixed_v_records(index, torch.zeros((1, 1), dtype=torch.int32))
    payload[0] |= 500 << 10
    with pytest.raises(ValueError, match="496"):
        unpack_mixed_v_records(payload, (1, 1))
    with pytest.raises(ValueError, match="10-bit"):
        pack_mixed_v_records(torch.full((1, 1), 1024, dtype=torch.int32), torch.zeros((1, 1), dtype=torch.int32))


def test_mixed_v_linear_equals_its_packed_layer_in_the_oracle() -> None:
    state = mixed_v_state(97, 50, 40, 3, seed=5, bias=True, outliers=2)
    packed = state.to_packed()
    x = np.random.default_rng(0).standard_normal((4, 97)).astype(np.float32)
    layer = po.OracleLayer(
        97, 50, 40, packed.left_words.numpy(), packed.right_words.numpy(), packed.scale_pre.float().numpy(),
        packed.scale_mid.float().numpy(), packed.scale_post.float().numpy(), packed.bias.float().numpy(),
        packed.outlier_indices.numpy(), packed.outlier_values.numpy(), packed.outlier_scales.float().numpy())
    dense_v = po.unpack_signs(packed.right_words.numpy(), 40, 97)
    dense_u = po.unpack_signs(packed.left_words.numpy(), 50, 40)
    latent = (x * packed.scale_pre.float().numpy()) @ dense_v.T * packed.scale_mid.float().numpy()
    expected = latent @ dense_u.T * packed.scale_post.float().numpy() + packed.bias.float().numpy()
    w = packed.outlier_values.float().numpy() * packed.outlier_scales.float().numpy()
    expected += x[:, packed.outlier_indices.numpy()] @ w.T
    np.testing.assert_allclose(po.packed_linear(x, layer), expected, rtol=1e-4, atol=1e-5)


# ------------------------------------------------------------------ GPU ---


def _require_b200() -> None:
    if not torch.cuda.is_available():
        pytest.fail("GPU test needs CUDA")
    assert torch.cuda.get_device_capability() == (10, 0), "tests target sm_100 (B200)"


@pytest.mark.gpu
@pytest.mark.parametrize(("n", "r", "free_rows"), ((64, 7, 2), (97, 40, 1), (1152, 987, 1), (4096, 3072, 64)))
def test_device_decode_is_bit_exact(n: int, r: int, free_rows: int) -> None:
    _require_b200()
    from nanoquant_b200.device_ops import decode_mixed_v_cuda

    state = mixed_v_state(n, 32, r, free_rows, seed=r)
    words = decode_mixed_v_cuda(state.free_right_words.cuda(), state.coded_payload.cuda(),
                                state.codebook_words.cuda(), rank=r, columns=n)
    assert torch.equal(words.cpu(), state.to_packed().right_words)


@pytest.mark.gpu
@pytest.mark.parametrize("tensor_cores", (True, False))
def test_mixed_v_layer_on_every_path_matches_oracle(tensor_cores: bool) -> None:
    _require_b200()
    from nanoquant_b200 import CudaPackedSm100Backend, OutlierRowOverlay, OverlaidLayerState
    from nanoquant_b200.cuda_backend import kernel_path

    # Gemma-3-1B up-projection shape (1152 -> 6912, r = 987) with bias and salient columns
    state = mixed_v_state(1152, 6912, 987, 1, seed=3, bias=True, outliers=3)
    backend = CudaPackedSm100Backend(tensor_cores=tensor_cores)
    layer = backend.prepare(state, "cuda")
    packed = state.to_packed()
    oracle = po.OracleLayer(
        1152, 6912, 987, packed.left_words.numpy(), packed.right_words.numpy(), packed.scale_pre.float().numpy(),
        packed.scale_mid.float().numpy(), packed.scale_post.float().numpy(), packed.bias.float().numpy(),
        packed.outlier_indices.numpy(), packed.outlier_values.numpy(), packed.outlier_scales.float().numpy())
    g = torch.Generator().manual_seed(7)
    for tokens in (1, 5, 64):
        x = torch.randn(tokens, 1152, generator=g).bfloat16()
        got = backend.linear(x.cuda(), layer).cpu()
        expected = po.packed_linear(x.float().numpy(), oracle, accumulate="float64")
        err = float((got - torch.from_numpy(expected)).abs().max() / np.abs(expected).max())
        assert err <= 2e-3, (tokens, kernel_path(layer, tokens), err)
    # with an int8 residual-row overlay on 1 % of the rows
    rows = torch.sort(torch.randperm(6912, generator=g)[:70]).values.to(torch.int32)
    overlay = OutlierRowOverlay(rows, torch.randint(-127, 128, (70, 1152), generator=g, dtype=torch.int8),
                                torch.full((70,), 0.002, dtype=torch.float16))
    layer = backend.prepare(OverlaidLayerState(state, overlay), "cuda")
    oracle.overlay_row_ids = rows.numpy()
    oracle.overlay_values = overlay.values.numpy()
    oracle.overlay_scales = overlay.scales.float().numpy()
    x = torch.randn(3, 1152, generator=g).bfloat16()
    got = backend.linear(x.cuda(), layer).cpu()
    expected = po.packed_linear(x.float().numpy(), oracle, accumulate="float64")
    assert float((got - torch.from_numpy(expected)).abs().max() / np.abs(expected).max()) <= 2e-3
