"""CUDA parity: libnqb through the C ABI against the reference's outputs and the CPU oracle.

Tolerances: the reference's own GPU test bound ``rtol=2e-5, atol=2e-4`` against
an fp32 restatement (reference ``tests/unit/test_runtime_cuda_backend.py:491``)
on the small fixtures; bit-exact for every integer/bit path (pack, unpack,
codebook decode); bitwise replay determinism; and for large layers the
``max|y - y_ref| / max|y_ref| <= 2e-3`` accuracy bound of the operator.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from nanoquant_b200 import (
    PACKED_LAYOUT_VERSION,
    CudaPackedSm100Backend,
    LogicalLayerState,
    OutlierRowOverlay,
    OverlaidLayerState,
    PackedLayerState,
    ProductCodebookLayerState,
    QuantizedLinearSpec,
    WorkloadSpec,
    grouped_sm100_projection,
    pack_logical_layer,
    prepare_sm100_projection_group,
)
from nanoquant_b200.device_ops import decode_product_codebook_cuda, pack_signs_cuda, unpack_signs_cuda
from oracle import packed_oracle as po
from tests.fixtures import as_numpy_f32, linear_names, load

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-5, 2e-4
# Persistent decode programs quantise activations to 22-bit fixed point up to
# 2 tokens and to 14-bit from 3 tokens on (two int8 digits per token: fewer
# MMAs); the 14-bit outputs are bounded by 1e-3 of max|y|, inside the
# operator's 2e-3 bound (and measured near 1e-4).
PROGRAM_WIDE_BOUND = 1e-3


def program_tolerance(tokens: int, scale: float) -> tuple[float, float]:
    """(rtol, atol) for a program output of `tokens` tokens whose reference has max|y| = scale."""

    if tokens >= 3:
        return 0.0, PROGRAM_WIDE_BOUND * scale
    return RTOL, max(ATOL, 1e-5 * scale)


@pytest.fixture(scope="module", autouse=True)
def _require_b200() -> None:
    if not torch.cuda.is_available():
        pytest.fail("GPU test needs CUDA")
    assert torch.cuda.get_device_capability() == (10, 0), "tests target sm_100 (B200)"


def _dtype_name(value: torch.Tensor | None) -> str | None:
    return None if value is None else str(value.dtype).removeprefix("torch.")


def state_from_case(case: dict) -> PackedLayerState:
    n, m, r = int(case["in_features"]), int(case["out_features"]), int(case["rank"])
    indices = case.get("outlier_indices")
    values = case.get("outlier_values")
    spec = QuantizedLinearSpec(
        "blocks.0.linear", "nanoquant-v1", n, m, r, "float32", _dtype_name(case["scale_pre"]),
        outlier_count=0 if indices is None else int(indices.numel()),
        outlier_value_dtype=_dtype_name(values),
        has_outlier_scales=case.get("outlier_scales") is not None,
        has_bias=case.get("bias") is not None,
        patch_rank=0 if case.get("patch_left") is None else int(case["patch_left"].shape[1]),
        patch_value_dtype=_dtype_name(case.get("patch_left")),
        bias_dtype=None,
    )
    return PackedLayerState(
        spec, PACKED_LAYOUT_VERSION, case["left_words"], case["right_words"], case["scale_pre"],
        case["scale_mid"], case["scale_post"], case.get("bias"),
        None if indices is None else indices.to(torch.int32), values, case.get("outlier_scales"),
        case.get("patch_left"), case.get("patch_right"),
    )


def oracle_from_state(state: PackedLayerState) -> po.OracleLayer:
    def f(v):
        return None if v is None else v.float().numpy()

    return po.OracleLayer(
        state.spec.in_features, state.spec.out_features, state.spec.rank,
        state.left_words.numpy(), state.right_words.numpy(), f(state.scale_pre), f(state.scale_mid),
        f(state.scale_post), f(state.bias),
        None if state.outlier_indices is None else state.outlier_indices.numpy(),
        None if state.outlier_values is None else (
            state.outlier_values.numpy() if state.outlier_values.dtype == torch.int8 else f(state.outlier_values)),
        f(state.outlier_scales), f(state.patch_left), f(state.patch_right),
    )


@pytest.mark.parametrize("name", linear_names())
def test_linear_matches_reference_fixture(name: str) -> None:
    case = load(name)
    state = state_from_case(case)
    backend = CudaPackedSm100Backend()
    tokens = tuple(case["x"].shape[:-1])
    workload = WorkloadSpec("decode" if tokens == (1,) else "prefill", "cuda", _dtype_name(case["x"]),
                            tokens[0], 1 if len(tokens) == 1 else tokens[-1], deterministic=True)
    assert backend.supports(state.spec, workload).supported
    prepared = backend.prepare(state, "cuda")
    x = case["x"].cuda()
    actual = backend.linear(x, prepared)
    repeated = backend.linear(x, prepared)
    assert actual.dtype is torch.float32
    assert actual.shape == case["y"].shape
    torch.testing.assert_close(actual.cpu(), case["y"], rtol=RTOL, atol=ATOL)
    oracle = po.packed_linear(as_numpy_f32(case["x"]), oracle_from_state(state))
    torch.testing.assert_close(actual.cpu(), torch.from_numpy(oracle), rtol=RTOL, atol=ATOL)
    assert torch.equal(actual, repeated)


@pytest.mark.parametrize("columns", (1, 31, 32, 33, 65, 128))
def test_device_pack_and_unpack_are_bit_exact(columns: int) -> None:
    fixture = load("packing")
    signs = torch.from_numpy(fixture[f"signs_{columns}"]).cuda()
    words = pack_signs_cuda(signs)
    assert np.array_equal(words.cpu().numpy(), fixture[f"words_{columns}"])
    unpacked, bad = unpack_signs_cuda(words, 3, columns)
    assert torch.equal(unpacked.cpu(), signs.cpu())
    assert int(bad.item()) == 0


def test_device_unpack_counts_bad_padding() -> None:
    fixture = load("packing")
    words = torch.from_numpy(fixture["words_33"]).clone()
    words[1, -1] |= 4
    _, bad = unpack_signs_cuda(words.cuda(), 3, 33)
    assert int(bad.item()) == 1


def test_device_pack_large_matrix() -> None:
    fixture = load("packing")
    words = pack_signs_cuda(torch.from_numpy(fixture["big_signs"]).cuda().bfloat16())
    assert np.array_equal(words.cpu().numpy(), fixture["big_words"])


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
def test_product_codebook_matches_reference_and_expanded_layer(tag: str) -> None:
    fixture = load("product_codebook")
    state = _codebook_state(fixture, tag)
    x = fixture[f"{tag}_x"].cuda()
    # same kernels on the compact and the decoded layer: bitwise equal
    generic = CudaPackedSm100Backend(tensor_cores=False)
    compact_out = generic.linear(x, generic.prepare(state, "cuda"))
    expanded_out = generic.linear(x, generic.prepare(state.to_packed(), "cuda"))
    assert torch.equal(compact_out, expanded_out)
    torch.testing.assert_close(compact_out.cpu(), fixture[f"{tag}_y"], rtol=RTOL, atol=ATOL)
    backend = CudaPackedSm100Backend()
    default_out = backend.linear(x, backend.prepare(state, "cuda"))
    torch.testing.assert_close(default_out.cpu(), fixture[f"{tag}_y"], rtol=RTOL, atol=ATOL)


def test_product_codebook_layer_on_tensor_core_paths() -> None:
    """A compact codebook layer (C4 shape: Gemma-1B gate) takes the tensor-core decode and prefill paths."""

    from nanoquant_b200.cuda_backend import kernel_path
    from nanoquant_b200.program import DecodeProgram, ProgramOp

    fixture = load("product_codebook")
    state = _codebook_state(fixture, "c4like")
    n = state.spec.in_features
    backend = CudaPackedSm100Backend()
    layer = backend.prepare(state, "cuda")
    oracle = oracle_from_state(state.to_packed())
    g = torch.Generator().manual_seed(11)
    for tokens, path in ((1, "tensor-core"), (5, "tensor-core"), (64, "prefill")):
        assert kernel_path(layer, tokens) == path
        x = torch.randn(tokens, n, generator=g).bfloat16()
        got = backend.linear(x.cuda(), layer)
        expected = po.packed_linear(x.float().numpy(), oracle, accumulate="float64")
        bound = PREFILL_BOUND if path == "prefill" else 2e-5
        assert _relative_max_error(got, expected) <= bound
    x = torch.randn(1, n, generator=g).bfloat16().cuda()
    out = DecodeProgram([ProgramOp((layer,), x)]).run()[0][0]
    expected = po.packed_linear(x.float().cpu().numpy(), oracle, accumulate="float64")
    assert _relative_max_error(out, expected) <= 2e-5
    assert ctypes_status() == 0


def test_device_codebook_decode_is_bit_exact() -> None:
    fixture = load("product_codebook")
    n, m, r, free_rows, _ = (int(v) for v in fixture["c4like_shape"])
    words = decode_product_codebook_cuda(
        fixture["c4like_factor_right_free_words"].cuda(), fixture["c4like_factor_right_coded_payload"].cuda(),
        fixture["c4like_first_half_words"].cuda(), fixture["c4like_second_half_words"].cuda(), rank=r, columns=n,
    )
    assert torch.equal(words.cpu(), fixture["c4like_right_words"])


@pytest.mark.parametrize("count", (2, 3))
def test_grouped_projection_matches_individual_layers(count: int) -> None:
    backend = CudaPackedSm100Backend()
    cases = [load(f"grouped_{i}") for i in range(count)]
    prepared = tuple(backend.prepare(state_from_case(case), "cuda") for case in cases)
    group = prepare_sm100_projection_group(prepared)
    assert group is not None
    x = cases[0]["x"].cuda()
    actual = grouped_sm100_projection(x, group)
    individual = tuple(backend.linear(x, layer) for layer in prepared)
    for got, single, case in zip(actual, individual, cases, strict=True):
        torch.testing.assert_close(got, single, rtol=2e-5, atol=5e-5)
        torch.testing.assert_close(got.cpu(), case["y"], rtol=RTOL, atol=ATOL)


def _random_state(n: int, m: int, r: int, seed: int, *, outliers: int = 0, scale_dtype=torch.float16,
                  bias: bool = False) -> PackedLayerState:
    g = torch.Generator().manual_seed(seed)
    spec = QuantizedLinearSpec(
        "blocks.0.r", "nanoquant-v1", n, m, r, "float32", str(scale_dtype).removeprefix("torch."),
        outlier_count=outliers, outlier_value_dtype="int8" if outliers else None,
        has_outlier_scales=bool(outliers), has_bias=bias,
    )
    pre = (torch.randn(n, generator=g).abs() * 0.05 + 0.01).to(scale_dtype)
    idx = None
    if outliers:
        idx = torch.sort(torch.randperm(n, generator=g)[:outliers]).values
        pre[idx] = 0
    logical = LogicalLayerState(
        spec,
        torch.where(torch.rand(m, r, generator=g) > 0.5, 1.0, -1.0),
        torch.where(torch.rand(r, n, generator=g) > 0.5, 1.0, -1.0),
        pre,
        torch.ones(r).to(scale_dtype),
        (torch.randn(m, generator=g).abs() * 0.05 + 0.01).to(scale_dtype),
        bias=torch.randn(m, generator=g).to(scale_dtype) if bias else None,
        outlier_indices=idx,
        outlier_values=torch.randint(-127, 128, (m, outliers), generator=g, dtype=torch.int8) if outliers else None,
        outlier_scales=torch.full((outliers,), 0.002).to(scale_dtype) if outliers else None,
    )
    return pack_logical_layer(logical)


def _relative_max_error(actual: torch.Tensor, expected: np.ndarray) -> float:
    ref = torch.from_numpy(expected).float()
    return float((actual.cpu() - ref).abs().max() / ref.abs().max())


@pytest.mark.parametrize("tokens", (1, 2, 5, 8, 16))
@pytest.mark.parametrize(("n", "m", "r"), ((640, 2048, 480), (4096, 4096, 2048), (4096, 1024, 819), (12288, 4096, 3072)))
def test_large_layers_within_north_star_tolerance(n: int, m: int, r: int, tokens: int) -> None:
    state = _random_state(n, m, r, seed=n + m + r + tokens)
    backend = CudaPackedSm100Backend()
    prepared = backend.prepare(state, "cuda")
    g = torch.Generator().manual_seed(tokens)
    x = torch.randn(tokens, n, generator=g).bfloat16()
    actual = backend.linear(x.cuda(), prepared)
    expected = po.packed_linear(x.float().numpy(), oracle_from_state(state), accumulate="float64")
    assert _relative_max_error(actual, expected) <= 2e-3
    np.testing.assert_allclose(actual.cpu().numpy(), expected, rtol=1e-4, atol=1e-4 * np.abs(expected).max())
    assert torch.equal(actual, backend.linear(x.cuda(), prepared))


def test_row_overlay_matches_oracle() -> None:
    base = _random_state(1152, 6912, 987, seed=77, outliers=0)
    g = torch.Generator().manual_seed(5)
    rows = torch.sort(torch.randperm(6912, generator=g)[:70]).values.to(torch.int32)
    overlay = OutlierRowOverlay(rows, torch.randint(-127, 128, (70, 1152), generator=g, dtype=torch.int8),
                                torch.full((70,), 0.002, dtype=torch.float16))
    state = OverlaidLayerState(base, overlay)
    backend = CudaPackedSm100Backend()
    prepared = backend.prepare(state, "cuda")
    x = torch.randn(3, 1152, generator=g).bfloat16()
    actual = backend.linear(x.cuda(), prepared)
    layer = oracle_from_state(base)
    layer.overlay_row_ids = rows.numpy()
    layer.overlay_values = overlay.values.numpy()
    layer.overlay_scales = overlay.scales.float().numpy()
    expected = po.packed_linear(x.float().numpy(), layer, accumulate="float64")
    np.testing.assert_allclose(actual.cpu().numpy(), expected, rtol=1e-4, atol=1e-4 * np.abs(expected).max())


def test_contract_errors_match_reference_backend() -> None:
    case = load("linear_fixture_none_t1")
    backend = CudaPackedSm100Backend()
    prepared = backend.prepare(state_from_case(case), "cuda")
    x = case["x"].cuda()
    with pytest.raises(ValueError, match="same device"):
        backend.linear(case["x"], prepared)
    with pytest.raises(ValueError, match="feature dimension"):
        backend.linear(x[..., :-1].contiguous(), prepared)
    with pytest.raises(ValueError, match="contiguous"):
        backend.linear(torch.cat((x, x), dim=-1)[..., ::2], prepared)
    with pytest.raises(ValueError, match="autograd"):
        backend.linear(x.float().requires_grad_(), prepared)
    with pytest.raises(ValueError, match="dtype is unsupported"):
        backend.linear(x.to(torch.int32), prepared)


def test_cuda_graph_replay_matches_eager() -> None:
    state = _random_state(1152, 1152, 576, seed=8, outliers=4, bias=True)
    backend = CudaPackedSm100Backend()
    prepared = backend.prepare(state, "cuda")
    x = torch.randn(1, 1152, device="cuda").bfloat16()
    eager = backend.linear(x, prepared)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        backend.linear(x, prepared)
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = backend.linear(x, prepared)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(captured, eager)


# ------------------------------------------------------------------ tensor-core decode path ---

@pytest.mark.parametrize("tokens", (1, 3, 6, 11, 16))
@pytest.mark.parametrize(("n", "m", "r"), ((35, 17, 33), (640, 2048, 480), (1152, 1024, 542), (4096, 1024, 819),
                                           (6912, 1152, 987)))
def test_tensor_core_path_matches_generic_and_oracle(n: int, m: int, r: int, tokens: int) -> None:
    from nanoquant_b200.cuda_backend import kernel_path

    state = _random_state(n, m, r, seed=3 * n + m + tokens, outliers=3, bias=True)
    fast = CudaPackedSm100Backend()
    slow = CudaPackedSm100Backend(tensor_cores=False)
    fast_layer = fast.prepare(state, "cuda")
    slow_layer = slow.prepare(state, "cuda")
    assert kernel_path(fast_layer, tokens) == "tensor-core"
    assert kernel_path(slow_layer, tokens) == "generic"
    g = torch.Generator().manual_seed(tokens)
    x = torch.randn(tokens, n, generator=g).bfloat16()
    got = fast.linear(x.cuda(), fast_layer)
    reference = slow.linear(x.cuda(), slow_layer)
    expected = po.packed_linear(x.float().numpy(), oracle_from_state(state), accumulate="float64")
    scale = float(np.abs(expected).max())
    np.testing.assert_allclose(got.cpu().numpy(), expected, rtol=RTOL, atol=max(ATOL, 1e-5 * scale))
    np.testing.assert_allclose(got.cpu().numpy(), reference.cpu().numpy(), rtol=RTOL, atol=max(ATOL, 1e-5 * scale))
    assert torch.equal(got, fast.linear(x.cuda(), fast_layer))
    status = ctypes_status()
    assert status == 0


def ctypes_status() -> int:
    import ctypes

    from nanoquant_b200 import _native

    value = ctypes.c_int32(-1)
    _native.call("nqb_device_status", ctypes.byref(value))
    return value.value


def test_tensor_core_grouped_projection_matches_members() -> None:
    backend = CudaPackedSm100Backend()
    states = [_random_state(4096, width, rank, seed=90 + i) for i, (width, rank) in
              enumerate(((4096, 2048), (1024, 819), (1024, 819)))]
    prepared = tuple(backend.prepare(state, "cuda") for state in states)
    group = prepare_sm100_projection_group(prepared)
    x = torch.randn(2, 4096, device="cuda").bfloat16()
    outs = grouped_sm100_projection(x, group)
    for out, state in zip(outs, states, strict=True):
        expected = po.packed_linear(x.float().cpu().numpy(), oracle_from_state(state), accumulate="float64")
        np.testing.assert_allclose(out.cpu().numpy(), expected, rtol=RTOL, atol=1e-5 * np.abs(expected).max())


# ------------------------------------------------------------------ tensor-core prefill path ---

PREFILL_BOUND = 2e-3  # the operator's bound on max|y - y_ref| / max|y_ref| (fp16 activations)


@pytest.mark.parametrize(("n", "m", "r", "tokens"), ((35, 17, 33, 40), (640, 2048, 480, 17), (640, 2048, 480, 300),
                                                      (1152, 6912, 987, 129), (4096, 4096, 2048, 256)))
def test_prefill_path_matches_oracle(n: int, m: int, r: int, tokens: int) -> None:
    from nanoquant_b200.cuda_backend import kernel_path

    state = _random_state(n, m, r, seed=7 * n + tokens, outliers=3, bias=True)
    backend = CudaPackedSm100Backend()
    layer = backend.prepare(state, "cuda")
    assert kernel_path(layer, tokens) == "prefill"
    g = torch.Generator().manual_seed(tokens)
    x = torch.randn(tokens, n, generator=g).bfloat16()
    got = backend.linear(x.cuda(), layer)
    expected = po.packed_linear(x.float().numpy(), oracle_from_state(state), accumulate="float64")
    assert _relative_max_error(got, expected) <= PREFILL_BOUND
    assert torch.equal(got, backend.linear(x.cuda(), layer))
    assert ctypes_status() == 0


@pytest.mark.parametrize(("scale_dtype", "x_dtype"), ((torch.bfloat16, torch.bfloat16), (torch.float32, torch.float32),
                                                      (torch.float16, torch.float16), (torch.float16, torch.float32)))
def test_prefill_scale_and_input_dtypes(scale_dtype: torch.dtype, x_dtype: torch.dtype) -> None:
    """fp16 pre scales are folded into the sign expansion; other dtypes are applied in the pre-pass."""

    from nanoquant_b200.cuda_backend import kernel_path

    state = _random_state(1152, 2048, 700, seed=5, outliers=2, bias=True, scale_dtype=scale_dtype)
    backend = CudaPackedSm100Backend()
    layer = backend.prepare(state, "cuda")
    assert kernel_path(layer, 96) == "prefill"
    x = torch.randn(96, 1152, generator=torch.Generator().manual_seed(3)).to(x_dtype)
    got = backend.linear(x.cuda(), layer)
    expected = po.packed_linear(x.float().numpy(), oracle_from_state(state), accumulate="float64")
    assert _relative_max_error(got, expected) <= PREFILL_BOUND
    assert ctypes_status() == 0


@pytest.mark.parametrize("n", (16416, 33000))
def test_prefill_rows_longer_than_the_row_pre_pass(n: int) -> None:
    """Wide rows: 256 threads per row (16416), and past 32768 columns the warp-per-token pre-pass (pre not folded)."""

    state = _random_state(n, 160, 96, seed=9)
    backend = CudaPackedSm100Backend()
    layer = backend.prepare(state, "cuda")
    x = torch.randn(20, n, generator=torch.Generator().manual_seed(4)).bfloat16()
    got = backend.linear(x.cuda(), layer)
    expected = po.packed_linear(x.float().numpy(), oracle_from_state(state), accumulate="float64")
    assert _relative_max_error(got, expected) <= PREFILL_BOUND
    assert ctypes_status() == 0


def test_prefill_grouped_qkv_with_unaligned_ranks() -> None:
    """Three members whose ranks are not multiples of 4: padded latent offsets, one TMA store map each."""

    backend = CudaPackedSm100Backend()
    states = (_random_state(1024, 1024, 450, seed=41), _random_state(1024, 256, 113, seed=42),
              _random_state(1024, 256, 113, seed=43))
    group = prepare_sm100_projection_group(tuple(backend.prepare(s, "cuda") for s in states))
    x = torch.randn(300, 1024, generator=torch.Generator().manual_seed(5)).bfloat16()
    outs = grouped_sm100_projection(x.cuda(), group)
    for got, state in zip(outs, states):
        expected = po.packed_linear(x.float().numpy(), oracle_from_state(state), accumulate="float64")
        assert _relative_max_error(got, expected) <= PREFILL_BOUND
    assert ctypes_status() == 0


def test_prefill_grouped_projection_and_overlay() -> None:
    backend = CudaPackedSm100Backend()
    base = _random_state(1152, 6912, 987, seed=31)
    g = torch.Generator().manual_seed(2)
    rows = torch.sort(torch.randperm(6912, generator=g)[:70]).values.to(torch.int32)
    overlay = OutlierRowOverlay(rows, torch.randint(-127, 128, (70, 1152), generator=g, dtype=torch.int8),
                                torch.full((70,), 0.002, dtype=torch.float16))
    up = _random_state(1152, 6912, 987, seed=32)
    layers = (backend.prepare(OverlaidLayerState(base, overlay), "cuda"), backend.prepare(up, "cuda"))
    group = prepare_sm100_projection_group(layers)
    x = torch.randn(64, 1152, generator=g).bfloat16()
    gate_out, up_out = grouped_sm100_projection(x.cuda(), group)
    gate_ref = oracle_from_state(base)
    gate_ref.overlay_row_ids = rows.numpy()
    gate_ref.overlay_values = overlay.values.numpy()
    gate_ref.overlay_scales = overlay.scales.float().numpy()
    for got, ref in ((gate_out, gate_ref), (up_out, oracle_from_state(up))):
        expected = po.packed_linear(x.float().numpy(), ref, accumulate="float64")
        assert _relative_max_error(got, expected) <= PREFILL_BOUND


def test_prepared_layers_hold_tiles_only_unless_asked() -> None:
    """After the tile copies are made the layout-v1 words leave the device; results do not change."""

    state = _random_state(640, 384, 200, seed=11, outliers=2, bias=True)
    lean = CudaPackedSm100Backend().prepare(state, "cuda")
    full = CudaPackedSm100Backend(keep_words=True).prepare(state, "cuda")
    assert not lean.payload.desc.left_words and not lean.payload.desc.right_words
    assert "left_words" not in lean.payload.tensors and "right_words" not in lean.payload.tensors
    assert full.payload.desc.left_words and full.payload.desc.right_words
    backend = CudaPackedSm100Backend()
    g = torch.Generator().manual_seed(11)
    for tokens in (1, 7, 40):
        x = torch.randn(tokens, 640, generator=g).bfloat16().cuda()
        assert torch.equal(backend.linear(x, lean), backend.linear(x, full))
    assert ctypes_status() == 0
