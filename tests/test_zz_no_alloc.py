"""nqb_linear_noalloc: the allocation-free entry point, checked against nqb_linear.

Some callers cannot allocate device memory: a plugin inside another engine's
executor, or a process with a fixed device-memory plan.  They call
``nqb_linear_noalloc``, which takes its scratch from a static array in the
library instead of a caller workspace.  This test calls it through the C ABI
twice in a row and compares each result with the existing entry point's
(``nqb_linear``, via the backend), within the parity tolerance of the other
GPU tests.  It also checks that a request larger than the static scratch is
refused without launching anything.  The file name sorts last so a run that
stops at the first failure has already run every other test.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from nanoquant_b200 import CudaPackedSm100Backend, _native
from nanoquant_b200.cuda_backend import kernel_path
from nanoquant_b200.decode_chain import random_packed_layer

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-5, 2e-4


@pytest.fixture(scope="module", autouse=True)
def _require_gpu() -> None:
    if not torch.cuda.is_available():
        pytest.fail("GPU test needs CUDA")


def _noalloc(layer, x: torch.Tensor) -> torch.Tensor:
    spec = layer.spec
    tokens = x.numel() // spec.in_features
    y = torch.empty((tokens, spec.out_features), dtype=torch.float32, device=x.device)
    _native.call(
        "nqb_linear_noalloc",
        ctypes.byref(layer.payload.desc),
        x.data_ptr(),
        _native.dtype_code(x.dtype),
        tokens,
        y.data_ptr(),
        _native.current_stream_handle(x.device),
    )
    return y


@pytest.mark.parametrize(("n", "m", "tokens"), ((4096, 4096, 1), (4096, 1024, 5), (1152, 6912, 16), (640, 2048, 24)))
def test_noalloc_matches_workspace_entry_point_twice(n: int, m: int, tokens: int) -> None:
    device = torch.device("cuda", torch.cuda.current_device())
    generator = torch.Generator(device=device).manual_seed(n + m + tokens)
    state = random_packed_layer("blocks.0.proj", n, m, m * n // (m + n), generator, device)
    backend = CudaPackedSm100Backend()
    layer = backend.prepare(state, device)
    expected_path = "tensor-core" if tokens <= 16 else "prefill"
    assert kernel_path(layer, tokens) == expected_path
    for call in range(2):
        x = torch.randn(tokens, n, device=device, generator=generator).bfloat16()
        got = _noalloc(layer, x)
        expected = backend.linear(x, layer)
        torch.cuda.synchronize()
        torch.testing.assert_close(got, expected, rtol=RTOL, atol=ATOL, msg=f"call {call}")


def test_noalloc_rejects_requests_beyond_its_static_scratch() -> None:
    device = torch.device("cuda", torch.cuda.current_device())
    generator = torch.Generator(device=device).manual_seed(1)
    state = random_packed_layer("blocks.0.proj", 4096, 4096, 2048, generator, device)
    layer = CudaPackedSm100Backend().prepare(state, device)
    tokens = 4096  # latent alone is 4096 * 2048 * 4 B = 32 MiB
    x = torch.zeros(tokens, 4096, device=device, dtype=torch.bfloat16)
    y = torch.full((tokens, 4096), 7.0, device=device)
    lib = _native.library()
    status = lib.nqb_linear_noalloc(ctypes.byref(layer.payload.desc), x.data_ptr(), _native.NQB_BF16, tokens,
                                    y.data_ptr(), _native.current_stream_handle(device))
    assert status == _native.NQB_ERR_WORKSPACE
    assert "static scratch" in lib.nqb_last_error().decode()
    torch.cuda.synchronize()
    assert bool((y == 7.0).all())  # nothing was launched
