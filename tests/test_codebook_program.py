"""Product-codebook layers in decode programs: V's coded rows stream as 16-bit records and decode in stage 1.

With ``coded_product_codebook=True``, ``prepare`` keeps, next to the expanded
sign tiles, coded tiles of V (``nqb_repack_product_codebook``): per 128-row
tile and 256-column slice, each row's 8 records (one per 32-column word) as a
16-byte block, and a 1024-word table (the first half words, then the second
half words shifted to bits 16..31).  A program streams those slices (2048
bytes instead of 4096) and each consumer lane decodes its own four sign words
(``table[rec & 255] | table[256 + (rec >> 8)]``, the record decode of
``product_codebook.py:110-143`` in the reference) where it would have loaded
them.  The decoded words are the expanded layer's words, so a program over
coded layers must give bitwise the outputs of the same program over the
expanded layers; both are also checked against the oracle.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from nanoquant_b200 import CudaPackedSm100Backend, QuantizedLinearSpec
from nanoquant_b200.packed import packed_word_count
from nanoquant_b200.product_codebook import (
    PRODUCT_CODEBOOK_FORMAT_VERSION,
    ProductCodebookLayerState,
    pack_product_codebook_indices,
)
from nanoquant_b200.program import DecodeProgram, ProgramOp
from oracle import packed_oracle as po
from tests.test_cuda_parity import ctypes_status, oracle_from_state, program_tolerance

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _require_gpu() -> None:
    if not torch.cuda.is_available():
        pytest.fail("GPU test needs CUDA")


def codebook_state(n: int, m: int, r: int, free_rows: int, seed: int) -> ProductCodebookLayerState:
    """A random canonical product-codebook layer: distinct half tables, uniform records, zero signs past n."""

    rng = np.random.default_rng(seed)
    wpr = packed_word_count(n)
    left = rng.integers(0, 2**32, size=(m, packed_word_count(r)), dtype=np.uint64).astype(np.uint32)
    if r % 32:
        left[:, -1] &= np.uint32((1 << (r % 32)) - 1)
    first = rng.integers(0, 2**16, size=256, dtype=np.uint32).astype(np.uint16)
    second = rng.integers(0, 2**16, size=256, dtype=np.uint32).astype(np.uint16)
    # the tail word's groups must decode to zero past column n: give them
    # records whose table entries are masked (entry 0 of each table cleared)
    first[0] = second[0] = 0
    records = rng.integers(0, 2**16, size=(r - free_rows, wpr), dtype=np.uint32)
    if n % 32:
        records[:, -1] = 0
    free = rng.integers(0, 2**32, size=(free_rows, wpr), dtype=np.uint64).astype(np.uint32)
    if n % 32:
        free[:, -1] &= np.uint32((1 << (n % 32)) - 1)
    half = lambda t: torch.from_numpy(t.view(np.int16).copy())  # noqa: E731
    scales = lambda k: torch.from_numpy((np.abs(rng.standard_normal(k)) * 0.05 + 0.01).astype(np.float16))  # noqa
    spec = QuantizedLinearSpec(f"blocks.0.cb{n}x{m}", "nanoquant-v1", n, m, r, "float32", "float16")
    return ProductCodebookLayerState(
        spec, PRODUCT_CODEBOOK_FORMAT_VERSION, False, free_rows,
        torch.from_numpy(left.view(np.int32).copy()), torch.from_numpy(free.view(np.int32).copy()),
        pack_product_codebook_indices(torch.from_numpy(records.astype(np.int32))), half(first), half(second),
        scales(n), scales(r), scales(m))


def _coded_tiles_reference(state: ProductCodebookLayerState) -> bytes:
    """The coded-tile bytes restated on the CPU from the record stream."""

    n, r, free_rows = state.spec.in_features, state.spec.rank, state.free_rows
    wpr = packed_word_count(n)
    slices = (wpr + 7) // 8
    first_tile = (free_rows + 127) // 128
    records = state.factor_right_coded_payload.numpy().view(np.uint16)
    out = bytearray()
    for t in range((r + 127) // 128 - first_tile):
        for s in range(slices):
            for row_in_tile in range(128):
                row = (first_tile + t) * 128 + row_in_tile
                block = np.zeros(8, dtype=np.uint16)
                for j in range(8):
                    w = 8 * s + j
                    if row < r and w < wpr:
                        block[j] = records[(row - free_rows) * wpr + w]
                out += block.tobytes()
    return bytes(out)


@pytest.mark.parametrize(("n", "r", "free_rows"), ((96, 200, 1), (700, 300, 37), (1152, 987, 128), (512, 400, 129)))
def test_coded_tiles_match_the_cpu_repack(n: int, r: int, free_rows: int) -> None:
    from nanoquant_b200.device_ops import repack_product_codebook_cuda

    state = codebook_state(n, 32, r, free_rows, seed=r + n)
    tiles, table = repack_product_codebook_cuda(
        state.factor_right_coded_payload.cuda(), state.first_half_words.cuda(), state.second_half_words.cuda(),
        rank=r, columns=n, free_rows=free_rows)
    expected = _coded_tiles_reference(state)
    assert bytes(tiles.cpu().numpy()[: len(expected)]) == expected
    first = state.first_half_words.numpy().view(np.uint16).astype(np.uint32)
    second = state.second_half_words.numpy().view(np.uint16).astype(np.uint32)
    want = np.concatenate((first, second << 16, np.zeros(512, dtype=np.uint32)))
    assert np.array_equal(table.cpu().numpy().view(np.uint32), want)


def _check(got: torch.Tensor, x: torch.Tensor, state: ProductCodebookLayerState) -> None:
    expected = po.packed_linear(x.float().cpu().numpy(), oracle_from_state(state.to_packed()), accumulate="float64")
    rtol, atol = program_tolerance(x.numel() // x.shape[-1], float(np.abs(expected).max()))
    np.testing.assert_allclose(got.cpu().numpy(), expected, rtol=rtol, atol=atol)


@pytest.mark.parametrize("tokens", (1, 2, 5, 16))
def test_program_over_codebook_layers_equals_the_expanded_program(tokens: int) -> None:
    from tests.test_cuda_parity import _random_state

    # a QKV-like op (two codebook members around a plain one; free rows inside,
    # at and past the first tile) and an op reading the first member's output
    qkv_states = [codebook_state(1152, 1024, 987, 37, seed=1), _random_state(1152, 256, 200, seed=2),
                  codebook_state(1152, 256, 300, 128, seed=3)]
    o_state = codebook_state(1024, 1152, 640, 129, seed=4)
    x = torch.randn(tokens, 1152, generator=torch.Generator().manual_seed(tokens)).bfloat16().cuda()

    def build(coded: bool):
        backend = CudaPackedSm100Backend(coded_product_codebook=coded)
        qkv = tuple(backend.prepare(s, "cuda") for s in qkv_states)
        o_proj = backend.prepare(o_state, "cuda")
        q = torch.empty(tokens, 1024, device="cuda")
        outs = [(q, torch.empty(tokens, 256, device="cuda"), torch.empty(tokens, 256, device="cuda")),
                (torch.empty(tokens, 1152, device="cuda"),)]
        program = DecodeProgram([ProgramOp(qkv, x), ProgramOp((o_proj,), q)], outputs=outs)
        return program, qkv

    coded, qkv = build(True)
    assert qkv[0].payload.desc.coded_right_tiles and not qkv[1].payload.desc.coded_right_tiles
    plain, plain_qkv = build(False)
    assert not plain_qkv[0].payload.desc.coded_right_tiles
    got = [t.clone() for op in coded.run() for t in op]
    ref = [t.clone() for op in plain.run() for t in op]
    torch.cuda.synchronize()
    for a, b in zip(got, ref):
        assert torch.equal(a, b)
    _check(got[0], x, qkv_states[0])
    _check(got[2], x, qkv_states[2])
    _check(got[3], got[0], o_state)
    again = [t for op in coded.run() for t in op]
    torch.cuda.synchronize()
    assert all(torch.equal(a, b) for a, b in zip(got, again))
    assert ctypes_status() == 0


@pytest.mark.parametrize("tokens", (1, 16))
def test_config4_chain_with_coded_records_equals_the_expanded_chain(tokens: int) -> None:
    """Two Gemma-3-1B config-4 layers (int8 outlier rows, free row 0) through the program engine."""

    from nanoquant_b200.decode_chain import GEMMA3_1B, DecodeChain, make_codebook_layers

    blocks = make_codebook_layers(GEMMA3_1B, layers=2, seed=7)
    coded = DecodeChain(GEMMA3_1B, blocks, torch.device("cuda"), tokens=tokens,
                        backend=CudaPackedSm100Backend(coded_product_codebook=True))
    plain = DecodeChain(GEMMA3_1B, blocks, torch.device("cuda"), tokens=tokens)
    assert coded.blocks[0].o_proj.payload.desc.coded_right_tiles
    for name, value in coded.inputs.items():
        plain.inputs[name].copy_(value)
    a = [t.clone() for op in coded.program.run() for t in op]
    b = [t.clone() for op in plain.program.run() for t in op]
    torch.cuda.synchronize()
    assert len(a) == len(b) == 2 * 7 and all(torch.equal(u, v) for u, v in zip(a, b))
