"""Low-rank patch (``y += L (R x)``) applied inside ``nqb_linear``, grouped calls and programs.

The reference adds the patch with two ``F.linear`` calls after the packed
product (``runtime/cuda_backend.py:275-277``, ``runtime/reference.py:224-232``).
Here the descriptor carries the factors: on the tensor-core decode path and in
decode programs the patch latent is formed in stage 1 and added in stage 2's
epilogue; the prefill and generic paths add it with two small kernels.  Every
path is compared with the float64 oracle (which applies the patch the
reference's way) within the decode tolerance of the packed product.
"""

from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch

from nanoquant_b200 import CudaPackedSm100Backend, _native, grouped_sm100_projection, prepare_sm100_projection_group
from nanoquant_b200.packed import PackedLayerState
from nanoquant_b200.program import DecodeProgram, ProgramOp
from oracle import packed_oracle as po
from tests.test_cuda_parity import (ATOL, PREFILL_BOUND, RTOL, _random_state, _relative_max_error, ctypes_status,
                                    program_tolerance,
                                    oracle_from_state)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _require_gpu() -> None:
    if not torch.cuda.is_available():
        pytest.fail("GPU test needs CUDA")


def _patched(n: int, m: int, r: int, p: int, seed: int, dtype: torch.dtype = torch.bfloat16,
             **kwargs) -> PackedLayerState:
    state = _random_state(n, m, r, seed=seed, **kwargs)
    g = torch.Generator().manual_seed(seed + 1000)
    spec = dataclasses.replace(state.spec, patch_rank=p, patch_value_dtype=str(dtype).removeprefix("torch."))
    left = (torch.randn(m, p, generator=g) * 0.05).to(dtype)
    right = (torch.randn(p, n, generator=g) * 0.05).to(dtype)
    return dataclasses.replace(state, spec=spec, patch_left=left, patch_right=right)


def _check(got: torch.Tensor, x: torch.Tensor, state: PackedLayerState, program: bool = False) -> None:
    """``program``: `got` comes from a decode program (14-bit activations from 3 tokens on)."""

    expected = po.packed_linear(x.float().cpu().numpy(), oracle_from_state(state), accumulate="float64")
    if x.numel() // x.shape[-1] > 16:
        # prefill path: fp16 activations, checked like every prefill result; its error must also stay far
        # below the patch's own size, or a dropped patch could pass
        assert _relative_max_error(got, expected) <= PREFILL_BOUND
        if state.patch_left is not None:
            error = float(np.abs(got.cpu().numpy() - expected).max())
            assert error < 0.1 * float(np.abs(_patch_only(x, state)).max())
        return
    rtol, atol = program_tolerance(x.numel() // x.shape[-1] if program else 1, float(np.abs(expected).max()))
    np.testing.assert_allclose(got.cpu().numpy(), expected, rtol=rtol, atol=atol)


def _patch_only(x: torch.Tensor, state: PackedLayerState) -> np.ndarray:
    xr = x.double().cpu().numpy() @ state.patch_right.double().numpy().T
    return xr @ state.patch_left.double().numpy().T


@pytest.mark.parametrize("dtype", (torch.bfloat16, torch.float32))
@pytest.mark.parametrize("tokens", (1, 5, 16, 40))
def test_patched_linear_matches_oracle(tokens: int, dtype: torch.dtype) -> None:
    # tokens 1..16 take the tensor-core decode path (patch fused), 40 the prefill path
    state = _patched(1024, 1536, 640, 24, seed=tokens, dtype=dtype, bias=True)
    backend = CudaPackedSm100Backend()
    layer = backend.prepare(state, "cuda")
    x = torch.randn(tokens, 1024, generator=torch.Generator().manual_seed(7)).bfloat16().cuda()
    got = backend.linear(x, layer)
    torch.cuda.synchronize()
    _check(got, x, state)
    # the patch is really there: it moves the result by far more than the tolerance
    assert float(np.abs(_patch_only(x, state)).max()) > 1e-2
    assert torch.equal(got, backend.linear(x, layer))  # deterministic
    assert ctypes_status() == 0


def test_patch_rank_above_the_stage_one_cta_count() -> None:
    # 300 patch rows over the few stage-1 CTAs of a small layer: each CTA forms several
    state = _patched(512, 640, 128, 300, seed=3)
    backend = CudaPackedSm100Backend()
    layer = backend.prepare(state, "cuda")
    for tokens in (1, 9):
        x = torch.randn(tokens, 512, generator=torch.Generator().manual_seed(tokens)).bfloat16().cuda()
        _check(backend.linear(x, layer), x, state)
    assert ctypes_status() == 0


def test_patched_linear_on_the_generic_path() -> None:
    state = _patched(320, 200, 96, 12, seed=5, dtype=torch.float16)
    backend = CudaPackedSm100Backend(tensor_cores=False)
    layer = backend.prepare(state, "cuda")
    x = torch.randn(3, 320, generator=torch.Generator().manual_seed(2)).cuda()
    _check(backend.linear(x, layer), x, state)
    assert ctypes_status() == 0


@pytest.mark.parametrize("tokens", (1, 7, 33))
def test_grouped_call_with_patched_members(tokens: int) -> None:
    states = [_patched(1024, 1024, 512, 16, seed=20), _random_state(1024, 256, 200, seed=21),
              _patched(1024, 256, 200, 40, seed=22, outliers=3)]
    backend = CudaPackedSm100Backend()
    layers = tuple(backend.prepare(s, "cuda") for s in states)
    group = prepare_sm100_projection_group(layers)
    assert group is not None
    x = torch.randn(tokens, 1024, generator=torch.Generator().manual_seed(tokens)).bfloat16().cuda()
    for got, state in zip(grouped_sm100_projection(x, group), states):
        _check(got, x, state)
    assert ctypes_status() == 0


@pytest.mark.parametrize("tokens", (1, 4, 16))
def test_program_with_patched_layers(tokens: int) -> None:
    backend = CudaPackedSm100Backend()
    qkv_states = [_patched(1024, 1024, 512, 32, seed=30), _random_state(1024, 256, 200, seed=31),
                  _patched(1024, 256, 200, 8, seed=32)]
    o_state = _patched(1024, 1024, 512, 200, seed=33, outliers=2, bias=True)
    qkv = tuple(backend.prepare(s, "cuda") for s in qkv_states)
    o_proj = backend.prepare(o_state, "cuda")
    x = torch.randn(tokens, 1024, generator=torch.Generator().manual_seed(tokens)).bfloat16().cuda()
    q = torch.empty(tokens, 1024, device="cuda")
    outputs = [(q, torch.empty(tokens, 256, device="cuda"), torch.empty(tokens, 256, device="cuda")),
               (torch.empty(tokens, 1024, device="cuda"),)]
    program = DecodeProgram([ProgramOp(qkv, x), ProgramOp((o_proj,), q)], outputs=outputs)
    results = program.run()
    torch.cuda.synchronize()
    for got, state in zip(results[0], qkv_states):
        _check(got, x, state, program=True)
    _check(results[1][0], q, o_state, program=True)
    first = [t.clone() for op in results for t in op]
    again = [t for op in program.run() for t in op]
    torch.cuda.synchronize()
    assert all(torch.equal(a, b) for a, b in zip(first, again))
    # the per-call path agrees to the same tolerance
    per_call = backend.linear(q, o_proj)
    rtol, atol = program_tolerance(tokens, float(per_call.abs().max()))
    torch.testing.assert_close(results[1][0], per_call, rtol=rtol, atol=atol)
    assert ctypes_status() == 0


def test_program_refuses_a_patched_swiglu_input() -> None:
    backend = CudaPackedSm100Backend()
    down = backend.prepare(_patched(1024, 640, 480, 8, seed=40), "cuda")
    gate = torch.zeros(1, 1024, device="cuda")
    with pytest.raises(_native.NativeError) as info:
        DecodeProgram([ProgramOp((down,), gate, x2=torch.zeros_like(gate))])
    assert info.value.status == _native.NQB_ERR_UNSUPPORTED
