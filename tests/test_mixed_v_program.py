"""Mixed-V layers in decode programs: V's coded rows stream as 19-bit records and decode in stage 1.

``prepare`` keeps, next to the expanded sign tiles, coded tiles of V
(``nqb_repack_mixed_v``): per 128-row tile and 256-column slice, each row's 8
records widened to 20 bits (codebook index | a << 10 | b << 15, the pair id
resolved) back to back from bit 160 r.  A program streams those (2560 bytes
per slice instead of 4096) and each consumer lane decodes its own four sign
words (codebook word with bits a and b flipped) where it would have loaded
them.  The decoded words
are the expanded layer's words, so a program over mixed-V layers must give
bitwise the outputs of the same program over their expanded packed layers;
both are also checked against the oracle.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from nanoquant_b200 import CudaPackedSm100Backend
from nanoquant_b200.mixed_v import MixedVLayerState, mixed_v_correction_pair_table
from nanoquant_b200.program import DecodeProgram, ProgramOp
from oracle import packed_oracle as po
from tests.test_cuda_parity import ATOL, RTOL, ctypes_status, oracle_from_state, program_tolerance
from tests.test_mixed_v import mixed_v_state

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _require_gpu() -> None:
    if not torch.cuda.is_available():
        pytest.fail("GPU test needs CUDA")


def _coded_tiles_reference(payload: np.ndarray, rank: int, n: int, free_rows: int) -> bytes:
    """The coded-tile bytes restated on the CPU from the record stream."""

    wpr = (n + 31) // 32
    slices = (wpr + 7) // 8
    first = (free_rows + 127) // 128
    tiles = (rank + 127) // 128 - first
    stream = payload.view(np.uint32).astype(np.uint64)
    pairs = mixed_v_correction_pair_table().numpy()

    def record(index: int) -> int:
        bit = index * 19
        word, shift = bit >> 5, bit & 31
        value = int(stream[word]) >> shift
        if shift > 13:
            value |= int(stream[word + 1]) << (32 - shift)
        value &= 0x7FFFF
        pair = int(pairs[value >> 10])
        return (value & 1023) | ((pair & 0xFF) << 10) | (((pair >> 8) & 0xFF) << 15)

    out = bytearray()
    for t in range(tiles):
        for s in range(slices):
            for r in range(128):
                row = (first + t) * 128 + r
                acc = 0
                for j in range(8):
                    w = 8 * s + j
                    if row < rank and w < wpr:
                        acc |= record((row - free_rows) * wpr + w) << (20 * j)
                out += acc.to_bytes(20, "little")
    return bytes(out)


@pytest.mark.parametrize(("n", "r", "free_rows"), ((97, 40, 1), (700, 300, 37), (1152, 987, 128), (512, 400, 129)))
def test_coded_tiles_match_the_cpu_repack(n: int, r: int, free_rows: int) -> None:
    from nanoquant_b200.device_ops import repack_mixed_v_cuda

    state = mixed_v_state(n, 32, r, free_rows, seed=r + n)
    got = repack_mixed_v_cuda(state.coded_payload.cuda(), rank=r, columns=n, free_rows=free_rows).cpu().numpy()
    expected = _coded_tiles_reference(state.coded_payload.numpy(), r, n, free_rows)
    assert bytes(got[: len(expected)]) == expected


def _check(got: torch.Tensor, x: torch.Tensor, state) -> None:
    if isinstance(state, MixedVLayerState):
        state = state.to_packed()
    expected = po.packed_linear(x.float().cpu().numpy(), oracle_from_state(state), accumulate="float64")
    rtol, atol = program_tolerance(x.numel() // x.shape[-1], float(np.abs(expected).max()))
    np.testing.assert_allclose(got.cpu().numpy(), expected, rtol=rtol, atol=atol)


@pytest.mark.parametrize("tokens", (1, 5, 16))
def test_program_over_mixed_v_layers_equals_the_expanded_program(tokens: int) -> None:
    backend = CudaPackedSm100Backend(coded_mixed_v=True)
    # a QKV-like op (two mixed-V members around a plain one; free rows inside,
    # at and past the first tile) and an op reading the first member's output
    from tests.test_cuda_parity import _random_state

    qkv_states = [mixed_v_state(1152, 1024, 987, 37, seed=1, bias=True),
                  _random_state(1152, 256, 200, seed=2),
                  mixed_v_state(1152, 256, 300, 128, seed=3, outliers=2)]
    o_state = mixed_v_state(1024, 1152, 640, 129, seed=4)
    x = torch.randn(tokens, 1152, generator=torch.Generator().manual_seed(tokens)).bfloat16().cuda()

    def build(expanded: bool):
        def prep(state):
            if expanded and isinstance(state, MixedVLayerState):
                state = state.to_packed()
            return backend.prepare(state, "cuda")

        qkv = tuple(prep(s) for s in qkv_states)
        o_proj = prep(o_state)
        q = torch.empty(tokens, 1024, device="cuda")
        outs = [(q, torch.empty(tokens, 256, device="cuda"), torch.empty(tokens, 256, device="cuda")),
                (torch.empty(tokens, 1152, device="cuda"),)]
        program = DecodeProgram([ProgramOp(qkv, x), ProgramOp((o_proj,), q)], outputs=outs)
        return program, qkv, o_proj

    coded, qkv, _ = build(False)
    assert qkv[0].payload.desc.coded_right_tiles and not qkv[1].payload.desc.coded_right_tiles
    plain, _, _ = build(True)
    got = [t.clone() for op in coded.run() for t in op]
    ref = [t.clone() for op in plain.run() for t in op]
    torch.cuda.synchronize()
    for a, b in zip(got, ref):
        assert torch.equal(a, b)
    for out, state in zip(got[:3], qkv_states):
        _check(out, x, state)
    _check(got[3], got[0], o_state)
    again = [t for op in coded.run() for t in op]
    torch.cuda.synchronize()
    assert all(torch.equal(a, b) for a, b in zip(got, again))
    assert ctypes_status() == 0


def test_coded_tiles_are_opt_in() -> None:
    state = mixed_v_state(640, 256, 300, 37, seed=9)
    assert not CudaPackedSm100Backend().prepare(state, "cuda").payload.desc.coded_right_tiles
    assert CudaPackedSm100Backend(coded_mixed_v=True).prepare(state, "cuda").payload.desc.coded_right_tiles

