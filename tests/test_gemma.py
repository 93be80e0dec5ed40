"""Gemma-3-1B decode step and its shell kernels against torch formulas and the oracle.

CPU tests pin the oracle's Gemma pieces (tanh GELU, sliding-window
attention) to torch.  ``gpu`` tests check the new shell kernels
(``nqb_embedding_bf16``, ``nqb_rmsnorm_residual`` with a normalised delta,
``nqb_decode_attention_window``), the gated-GELU program input, a two-layer
step, and the full config-1 step -- 26 layers, hidden 1152, MLP 6912, 4 q /
1 kv head of 256, 1024 cached tokens, local layers with a 512-key window --
against ``oracle.decoder_oracle.gemma_decode_step_streaming`` with the
full-model bound: cosine >= 0.9999 on the final hidden states.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import decoder_oracle as do


def test_oracle_gelu_tanh_matches_torch() -> None:
    x = np.linspace(-12, 12, 4001, dtype=np.float32)
    ref = torch.nn.functional.gelu(torch.from_numpy(x).double(), approximate="tanh").float().numpy()
    np.testing.assert_allclose(do.gelu_tanh(x), ref, rtol=1e-6, atol=1e-7)


def test_oracle_sliding_window_attention_matches_torch() -> None:
    rng = np.random.default_rng(3)
    q = rng.standard_normal((3, 4, 32)).astype(np.float32)
    kc = rng.standard_normal((1, 60, 32)).astype(np.float32)
    vc = rng.standard_normal((1, 60, 32)).astype(np.float32)
    out = do.attention(q, kc, vc, 50, window=16)
    for t in range(3):
        lo, hi = 50 + t - 16, 50 + t
        for h in range(4):
            s = torch.from_numpy(kc[0, lo:hi]).double() @ torch.from_numpy(q[t, h]).double() / np.sqrt(32)
            ref = torch.softmax(s, 0) @ torch.from_numpy(vc[0, lo:hi]).double()
            np.testing.assert_allclose(out[t, h], ref.numpy(), rtol=1e-5, atol=1e-6)


# ------------------------------------------------------------------ GPU ---


def _gpu() -> torch.device:
    if not torch.cuda.is_available():
        pytest.fail("GPU test needs CUDA")
    return torch.device("cuda", 0)


@pytest.mark.gpu
@pytest.mark.parametrize("dim", (1152, 1000))
def test_embedding_kernel(dim: int) -> None:
    from nanoquant_b200.decoder import embedding_bf16

    dev = _gpu()
    table = torch.randn(500, dim, device=dev).bfloat16()
    ids = torch.tensor([3, 499, 0, 7, 500, -1], dtype=torch.int64, device=dev)  # the last two are out of range
    out = torch.full((6, dim), 7.0, device=dev)
    embedding_bf16(ids, table, 34.0, out)
    torch.cuda.synchronize()
    assert torch.equal(out[:4], table[ids[:4]].float() * 34.0)
    assert torch.equal(out[4:], torch.zeros(2, dim, device=dev))


@pytest.mark.gpu
@pytest.mark.parametrize("hidden", (1152, 4096, 1000))
@pytest.mark.parametrize("tokens", (1, 5))
def test_rmsnorm_residual_normalises_the_delta(hidden: int, tokens: int) -> None:
    from nanoquant_b200.decoder import rmsnorm

    dev = _gpu()
    g = torch.Generator(device=dev).manual_seed(hidden + tokens)
    h = torch.randn(tokens, hidden, generator=g, device=dev)
    delta = torch.randn(tokens, hidden, generator=g, device=dev) * 3.0
    w = 1.0 + torch.randn(hidden, generator=g, device=dev) * 0.1
    dw = 1.0 + torch.randn(hidden, generator=g, device=dev) * 0.1
    out = torch.empty(tokens, hidden, device=dev)
    h64, d64 = h.double(), delta.double()
    new_h = h64 + d64 * torch.rsqrt(d64.pow(2).mean(-1, keepdim=True) + 1e-6) * dw.double()
    ref = new_h * torch.rsqrt(new_h.pow(2).mean(-1, keepdim=True) + 1e-6) * w.double()
    rmsnorm(h, delta, w, 1e-6, out, delta_weight=dw)
    torch.cuda.synchronize()
    torch.testing.assert_close(h.double(), new_h, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(out.double(), ref, rtol=1e-5, atol=1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize(("keys", "tokens", "window"), ((1025, 1, 512), (1025, 4, 512), (300, 2, 512), (70, 3, 16)))
def test_attention_window_matches_oracle(keys: int, tokens: int, window: int) -> None:
    from nanoquant_b200.decoder import attention_workspace_bytes, decode_attention

    dev = _gpu()
    g = torch.Generator(device=dev).manual_seed(keys + window)
    hd, hq, hkv = 256, 4, 1
    cache_len = keys + tokens - 1
    q = torch.randn(tokens, hq * hd, generator=g, device=dev).bfloat16()
    kc = torch.randn(hkv, cache_len, hd, generator=g, device=dev).bfloat16()
    vc = torch.randn(hkv, cache_len, hd, generator=g, device=dev).bfloat16()
    out = torch.empty(tokens, hq * hd, device=dev, dtype=torch.bfloat16)
    ws = torch.empty(attention_workspace_bytes(keys, tokens, hq, hd), dtype=torch.uint8, device=dev)
    decode_attention(q, kc, vc, keys, hq, hkv, hd, out, ws, window=window)
    torch.cuda.synchronize()
    ref = do.attention(q.float().cpu().numpy().reshape(tokens, hq, hd), kc.float().cpu().numpy(),
                       vc.float().cpu().numpy(), keys, window=window).reshape(tokens, hq * hd)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, rtol=1e-2, atol=1e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("tokens", (1, 5, 16))
def test_gated_gelu_program_input_matches_oracle(tokens: int) -> None:
    from nanoquant_b200 import CudaPackedSm100Backend
    from nanoquant_b200.program import DecodeProgram, ProgramOp
    from oracle import packed_oracle as po
    from tests.test_cuda_parity import _random_state, oracle_from_state

    dev = _gpu()
    backend = CudaPackedSm100Backend()
    down_state = _random_state(6912, 1152, 987, seed=91)
    down = backend.prepare(down_state, dev)
    g = torch.Generator(device=dev).manual_seed(tokens)
    gate = torch.randn(tokens, 6912, generator=g, device=dev) * 2.0
    up = torch.randn(tokens, 6912, generator=g, device=dev)
    out = torch.empty(tokens, 1152, device=dev)
    program = DecodeProgram([ProgramOp((down,), gate, x2=up, activation="gelu_tanh")], outputs=[(out,)])
    program.run()
    torch.cuda.synchronize()
    act = do.gelu_tanh(gate.cpu().numpy()) * up.cpu().numpy()
    ref = po.packed_linear(act, oracle_from_state(down_state), accumulate="float64")
    err = float(np.abs(out.cpu().numpy() - ref).max() / np.abs(ref).max())
    assert err <= (2e-5 if tokens < 3 else 1e-3), err  # programs: 14-bit activations from 3 tokens on


def _host_state(state):
    from dataclasses import fields, replace

    moved = {f.name: getattr(state, f.name).cpu() for f in fields(state)
             if isinstance(getattr(state, f.name), torch.Tensor)}
    return replace(state, **moved)


def _gemma_parity(shape, layers: int, tokens: int, position: int, seed: int) -> list[float]:
    """Cosines between the device step's final hidden states and the oracle's."""

    from nanoquant_b200.decode_chain import make_decoder_layers
    from nanoquant_b200.decoder import Gemma3DecodeStep, random_gemma_shell_weights
    from tests.test_cuda_parity import oracle_from_state

    dev = _gpu()
    blocks = make_decoder_layers(shape, dev, layers=layers, seed=seed)
    shell = random_gemma_shell_weights(shape, 4096, dev, layers=layers, seed=seed + 1)
    step = Gemma3DecodeStep(shape, blocks, shell, dev, tokens=tokens, position=position,
                            kv_init=torch.Generator(device=dev).manual_seed(seed + 2))
    ids = torch.randint(0, 4096, (tokens,), generator=torch.Generator().manual_seed(seed + 3)).to(dev)
    got = step.step(ids).cpu().numpy()
    caches = [(layer["k_cache"].float().cpu().numpy(), layer["v_cache"].float().cpu().numpy())
              for layer in step.layers]
    torch.cuda.synchronize()
    effective = lambda w: (1.0 + w.float()).cpu().numpy()  # noqa: E731

    def layer_at(i: int):
        proj = {name: oracle_from_state(_host_state(state)) for name, state in blocks[i].items()}
        norms = {"input_norm": effective(shell.input_norm[i]),
                 "post_attention_norm": effective(shell.post_attention_norm[i]),
                 "pre_feedforward_norm": effective(shell.pre_feedforward_norm[i]),
                 "post_feedforward_norm": effective(shell.post_feedforward_norm[i]),
                 "q_norm": effective(shell.q_norm[i]), "k_norm": effective(shell.k_norm[i])}
        return proj, norms, caches[i][0], caches[i][1]

    hidden = shell.embedding[ids].float().cpu().numpy() * step.embed_scale
    ref = do.gemma_decode_step_streaming(hidden, layers, layer_at, effective(shell.final_norm), position=position,
                                         q_heads=shape.q_heads, kv_heads=shape.kv_heads, head_dim=shape.head_dim,
                                         eps=1e-6, accumulate="float32")
    return [float(a.astype(np.float64) @ b / np.linalg.norm(a) / np.linalg.norm(b)) for a, b in zip(got, ref)]


@pytest.mark.gpu
@pytest.mark.parametrize("tokens", (1, 3))
def test_gemma_two_layer_step_matches_oracle(tokens: int) -> None:
    from nanoquant_b200.decode_chain import DecoderShape

    shape = DecoderShape("gemma-tiny", 6, 256, 512, 4, 1, 256, 1.0)
    cosines = _gemma_parity(shape, 6, tokens, position=40, seed=5)  # layer 5 is global, 0-4 local
    assert min(cosines) >= 0.9999, cosines


@pytest.mark.gpu
@pytest.mark.timeout(900)
def test_gemma3_1b_full_step_matches_oracle() -> None:
    from nanoquant_b200.decode_chain import GEMMA3_1B

    cosines = _gemma_parity(GEMMA3_1B, GEMMA3_1B.layers, 1, position=1024, seed=21)
    assert min(cosines) >= 0.9999, cosines


@pytest.mark.gpu
def test_gemma_step_graph_replay_is_bitwise_eager() -> None:
    from nanoquant_b200.decode_chain import DecoderShape
    from nanoquant_b200.decoder import build_gemma3_step

    dev = _gpu()
    shape = DecoderShape("gemma-tiny", 2, 256, 512, 4, 1, 256, 1.0)
    step = build_gemma3_step(shape, dev, vocab=1000, tokens=2, position=9, layers=2, seed=7)
    ids = torch.tensor([5, 17], device=dev)
    eager = step.step(ids).clone()
    step.capture()
    first = step.replay().clone()
    second = step.replay().clone()
    torch.cuda.synchronize()
    assert torch.equal(eager, first) and torch.equal(first, second)
