"""BASELINE config 4 at its own shapes: product-codebook V and 1 % int8 outlier rows on Gemma-3-1B projections.

Each 16-sign group of V is an 8-bit index into one per-layer table of 256
random 16-bit sign words (both half tables of ``product-codebook-free-k16-v1``
equal, row 0 the format's required free row); U is plain signs; 1 % of the
output rows carry an int8 residual row with fp16 scale 0.002.  CPU tests check
the builder against the format's definition; the ``gpu`` test runs every
projection of a layer at batch 1 (one persistent decode program) and at batch
64 (tensor-core prefill kernels) against the oracle: the codebook decoded to
layout v1 (``ProductCodebookLayerState.to_packed``, the reference's own
decode, ``product_codebook.py:229-269``) plus the row overlay restated from
its definition (parity unpinned for that form: the reference has no type for
it).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from nanoquant_b200.decode_chain import GEMMA3_1B, make_codebook_layers
from oracle import packed_oracle as po


def _oracle(state) -> po.OracleLayer:
    packed = state.base.to_packed()
    layer = po.OracleLayer(packed.spec.in_features, packed.spec.out_features, packed.spec.rank,
                           packed.left_words.numpy(), packed.right_words.numpy(), packed.scale_pre.float().numpy(),
                           packed.scale_mid.float().numpy(), packed.scale_post.float().numpy())
    layer.overlay_row_ids = state.overlay.row_ids.numpy()
    layer.overlay_values = state.overlay.values.numpy()
    layer.overlay_scales = state.overlay.scales.float().numpy()
    return layer


def test_builder_follows_the_config() -> None:
    (block,) = make_codebook_layers(GEMMA3_1B, layers=1, seed=3)
    for proj, (n, m) in GEMMA3_1B.projections().items():
        state = block[proj]
        base = state.base
        assert base.free_rows == 1 and torch.equal(base.first_half_words, base.second_half_words)
        assert state.overlay.row_ids.numel() == -(-m // 100)  # ceil(1 % of the rows)
        assert bool((state.overlay.scales.float() == np.float16(0.002)).all())
        assert int(state.overlay.values.abs().max()) <= 127
        # every V word (row 0 included) is first[lo] | second[hi] << 16 of the one table
        words = base.to_packed().right_words.numpy().view(np.uint32)
        table = base.first_half_words.numpy().view(np.uint16).astype(np.uint32)
        assert np.isin(words & 0xFFFF, table).all() and np.isin(words >> 16, table).all()


@pytest.mark.gpu
@pytest.mark.parametrize("tokens", (1, 64))
def test_config4_layer_matches_oracle(tokens: int) -> None:
    from nanoquant_b200 import CudaPackedSm100Backend
    from nanoquant_b200.cuda_backend import kernel_path
    from nanoquant_b200.program import DecodeProgram, ProgramOp

    if not torch.cuda.is_available():
        pytest.fail("GPU test needs CUDA")
    (block,) = make_codebook_layers(GEMMA3_1B, layers=1, seed=5)
    backend = CudaPackedSm100Backend()
    g = torch.Generator().manual_seed(tokens)
    for proj, state in block.items():
        prepared = backend.prepare(state, "cuda")
        x = torch.randn(tokens, state.spec.in_features, generator=g).bfloat16()
        if tokens == 1:
            program = DecodeProgram([ProgramOp((prepared,), x.cuda())])
            got = program.run()[0][0]
            bound = 2e-5
        else:
            assert kernel_path(prepared, tokens) == "prefill"
            got = backend.linear(x.cuda(), prepared)
            bound = 2e-3
        torch.cuda.synchronize()
        ref = po.packed_linear(x.float().numpy(), _oracle(state), accumulate="float64")
        err = float(np.abs(got.cpu().numpy() - ref).max() / np.abs(ref).max())
        assert err <= bound, (proj, err)
