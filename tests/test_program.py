"""Persistent decode program (``nqb_program_*``) against the oracle and the per-call path.

A program runs a fixed sequence of packed-linear calls in one cooperative
launch.  These tests build programs from the same layers as the per-call
tests, chain ops through each other's outputs (an op reads the fp32 output of
an earlier op, so the grid barriers must order them), and compare every output
with the float64 oracle within the tensor-core decode tolerance.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from nanoquant_b200 import (
    CudaPackedSm100Backend,
    OutlierRowOverlay,
    OverlaidLayerState,
    _native,
    grouped_sm100_projection,
    prepare_sm100_projection_group,
)
from nanoquant_b200.program import DecodeProgram, ProgramOp
from oracle import packed_oracle as po
from tests.test_cuda_parity import ATOL, RTOL, _random_state, ctypes_status, oracle_from_state, program_tolerance

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _require_gpu() -> None:
    if not torch.cuda.is_available():
        pytest.fail("GPU test needs CUDA")


def _check(got: torch.Tensor, x: torch.Tensor, state) -> None:
    expected = po.packed_linear(x.float().cpu().numpy(), oracle_from_state(state), accumulate="float64")
    rtol, atol = program_tolerance(x.numel() // state.spec.in_features, float(np.abs(expected).max()))
    np.testing.assert_allclose(got.cpu().numpy(), expected, rtol=rtol, atol=atol)


@pytest.mark.parametrize("tokens", (1, 3, 8, 11, 16))
def test_program_chain_matches_oracle(tokens: int) -> None:
    backend = CudaPackedSm100Backend()
    g = torch.Generator().manual_seed(tokens)
    qkv_states = [_random_state(4096, w, r, seed=10 + i) for i, (w, r) in enumerate(((4096, 2048), (1024, 819),
                                                                                       (1024, 819)))]
    o_state = _random_state(4096, 4096, 2048, seed=20, outliers=3, bias=True)
    gu_states = [_random_state(1152, 6912, 987, seed=30 + i) for i in range(2)]
    down_state = _random_state(6912, 1152, 987, seed=40, bias=True)
    qkv = tuple(backend.prepare(s, "cuda") for s in qkv_states)
    o_proj = backend.prepare(o_state, "cuda")
    gate_up = tuple(backend.prepare(s, "cuda") for s in gu_states)
    down = backend.prepare(down_state, "cuda")

    x0 = torch.randn(tokens, 4096, generator=g).bfloat16().cuda()
    x2 = torch.randn(tokens, 1152, generator=g).bfloat16().cuda()
    q_out = torch.empty(tokens, 4096, device="cuda")
    gate_out = torch.empty(tokens, 6912, device="cuda")
    ops = [
        ProgramOp(qkv, x0),
        ProgramOp((o_proj,), q_out),      # reads op 0's q output
        ProgramOp(gate_up, x2),
        ProgramOp((down,), gate_out),     # reads op 2's gate output
    ]
    outputs = [
        (q_out, torch.empty(tokens, 1024, device="cuda"), torch.empty(tokens, 1024, device="cuda")),
        (torch.empty(tokens, 4096, device="cuda"),),
        (gate_out, torch.empty(tokens, 6912, device="cuda")),
        (torch.empty(tokens, 1152, device="cuda"),),
    ]
    program = DecodeProgram(ops, outputs=outputs)
    assert program.ctas >= 4 and program.ctas % program.cluster_size == 0
    results = program.run()
    torch.cuda.synchronize()
    for got, state in zip(results[0], qkv_states):
        _check(got, x0, state)
    _check(results[1][0], q_out, o_state)
    for got, state in zip(results[2], gu_states):
        _check(got, x2, state)
    _check(results[3][0], gate_out, down_state)
    # the per-call tensor-core path on the same inputs agrees
    # (both round their 22-bit activation quantisation per K chunk, and the
    # chunks differ, so they agree to the same tolerance as with the oracle)
    per_call = grouped_sm100_projection(x0, prepare_sm100_projection_group(qkv)) + (backend.linear(q_out, o_proj),)
    for got, ref in zip((*results[0], results[1][0]), per_call):
        rtol, atol = program_tolerance(tokens, float(ref.abs().max()))
        torch.testing.assert_close(got, ref, rtol=rtol, atol=atol)
    assert ctypes_status() == 0


def test_program_is_deterministic_and_leaves_counters_zero() -> None:
    backend = CudaPackedSm100Backend()
    states = [_random_state(2048, 5632, 1500, seed=50 + i) for i in range(2)]
    layers = tuple(backend.prepare(s, "cuda") for s in states)
    x = torch.randn(2, 2048, generator=torch.Generator().manual_seed(1)).bfloat16().cuda()
    program = DecodeProgram([ProgramOp(layers, x), ProgramOp(layers[:1], x)])
    first = [tuple(t.clone() for t in op) for op in program.run()]
    second = program.run()
    torch.cuda.synchronize()
    for a_op, b_op in zip(first, second):
        for a, b in zip(a_op, b_op):
            assert torch.equal(a, b)
    assert int(program.workspace[:16384].count_nonzero()) == 0
    _check(second[1][0], x, states[0])
    assert ctypes_status() == 0


def test_program_applies_overlay_rows_and_salient_columns() -> None:
    backend = CudaPackedSm100Backend()
    base = _random_state(1152, 6912, 987, seed=61, outliers=4, bias=True)
    g = torch.Generator().manual_seed(2)
    rows = torch.sort(torch.randperm(6912, generator=g)[:70]).values.to(torch.int32)
    overlay = OutlierRowOverlay(rows, torch.randint(-127, 128, (70, 1152), generator=g, dtype=torch.int8),
                                torch.full((70,), 0.002, dtype=torch.float16))
    layer = backend.prepare(OverlaidLayerState(base, overlay), "cuda")
    x = torch.randn(5, 1152, generator=g).bfloat16().cuda()
    out = DecodeProgram([ProgramOp((layer,), x)]).run()[0][0]
    torch.cuda.synchronize()
    ref = oracle_from_state(base)
    ref.overlay_row_ids = rows.numpy()
    ref.overlay_values = overlay.values.numpy()
    ref.overlay_scales = overlay.scales.float().numpy()
    expected = po.packed_linear(x.float().cpu().numpy(), ref, accumulate="float64")
    rtol, atol = program_tolerance(x.shape[0], float(np.abs(expected).max()))
    np.testing.assert_allclose(out.cpu().numpy(), expected, rtol=rtol, atol=atol)
    assert ctypes_status() == 0


def test_program_rejects_prefill_token_counts() -> None:
    backend = CudaPackedSm100Backend()
    layer = backend.prepare(_random_state(640, 2048, 480, seed=70), "cuda")
    x = torch.zeros(17, 640, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_native.NativeError) as info:
        DecodeProgram([ProgramOp((layer,), x)])
    assert info.value.status == _native.NQB_ERR_UNSUPPORTED


@pytest.mark.parametrize("tokens", (1, 4, 16))
def test_program_swiglu_input_matches_oracle(tokens: int) -> None:
    """gate/up then down in one program: the down op forms silu(gate) * up as it loads its input."""

    backend = CudaPackedSm100Backend()
    gu_states = [_random_state(1152, 6912, 987, seed=80 + i) for i in range(2)]
    down_state = _random_state(6912, 1152, 987, seed=90, bias=True)
    gate_up = tuple(backend.prepare(s, "cuda") for s in gu_states)
    down = backend.prepare(down_state, "cuda")
    x = torch.randn(tokens, 1152, generator=torch.Generator().manual_seed(tokens)).bfloat16().cuda()
    gate = torch.empty(tokens, 6912, device="cuda")
    up = torch.empty(tokens, 6912, device="cuda")
    out = torch.empty(tokens, 1152, device="cuda")
    program = DecodeProgram([ProgramOp(gate_up, x), ProgramOp((down,), gate, x2=up)],
                            outputs=[(gate, up), (out,)])
    program.run()
    torch.cuda.synchronize()
    _check(gate, x, gu_states[0])
    _check(up, x, gu_states[1])
    act = torch.nn.functional.silu(gate) * up   # fp32, from the program's own gate/up outputs
    _check(out, act, down_state)
    assert ctypes_status() == 0


def test_program_swiglu_input_rejects_salient_columns_and_bad_x2() -> None:
    backend = CudaPackedSm100Backend()
    salient = backend.prepare(_random_state(1024, 640, 480, seed=95, outliers=2), "cuda")
    plain = backend.prepare(_random_state(1024, 640, 480, seed=96), "cuda")
    gate = torch.zeros(1, 1024, device="cuda")
    up = torch.zeros(1, 1024, device="cuda")
    with pytest.raises(_native.NativeError) as info:
        DecodeProgram([ProgramOp((salient,), gate, x2=up)])
    assert info.value.status == _native.NQB_ERR_UNSUPPORTED
    with pytest.raises(ValueError, match="fp32"):
        DecodeProgram([ProgramOp((plain,), gate.bfloat16(), x2=up.bfloat16())])
    with pytest.raises(ValueError, match="shaped like x"):
        DecodeProgram([ProgramOp((plain,), gate, x2=torch.zeros(2, 1024, device="cuda"))])


def _device_status() -> int:
    import ctypes

    status = ctypes.c_int32(-1)
    _native.call("nqb_device_status", ctypes.byref(status))
    return status.value


def test_program_grid_barrier_timeout_is_reported_and_recovered() -> None:
    """A grid barrier that cannot complete gives up, reports NQB_ERR_TIMEOUT and leaves the program reusable.

    The failure is made on the host: every barrier of the skewed run waits for
    one arrival more than the grid has CTAs, with a short poll limit, so each
    gives up after its limit instead of hanging.  The run's outputs are
    undefined; its workspace counters must be zero afterwards, and the next run
    on the same workspace must equal the run before it bit for bit.
    """

    backend = CudaPackedSm100Backend()
    states = [_random_state(1152, 6912, 987, seed=70 + i) for i in range(2)]
    down_state = _random_state(6912, 1152, 987, seed=72, bias=True)
    gate_up = tuple(backend.prepare(s, "cuda") for s in states)
    down = backend.prepare(down_state, "cuda")
    x = torch.randn(1, 1152, generator=torch.Generator().manual_seed(7)).bfloat16().cuda()
    gate = torch.empty(1, 6912, device="cuda")
    program = DecodeProgram([ProgramOp(gate_up, x), ProgramOp((down,), gate)],
                            outputs=[(gate, torch.empty(1, 6912, device="cuda")), (torch.empty(1, 1152, device="cuda"),)])
    assert _device_status() == _native.NQB_OK
    before = [t.clone() for op in program.run() for t in op]
    torch.cuda.synchronize()
    assert _device_status() == _native.NQB_OK

    _native.call("nqb_debug_set_barrier_limit", 1 << 12)
    _native.call("nqb_program_debug_barrier_skew", program._handle, 1)
    try:
        program.run()
        torch.cuda.synchronize()
        assert _device_status() == _native.NQB_ERR_TIMEOUT
        assert int(program.workspace[:16384].count_nonzero()) == 0
    finally:
        _native.call("nqb_program_debug_barrier_skew", program._handle, 0)
        _native.call("nqb_debug_set_barrier_limit", 0)

    after = [t.clone() for op in program.run() for t in op]
    torch.cuda.synchronize()
    assert _device_status() == _native.NQB_OK
    for a, b in zip(before, after):
        assert torch.equal(a, b)
