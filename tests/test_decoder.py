"""Decode-step shell (``nanoquant_b200.decoder``) against torch formulas and the decoder oracle.

CPU tests pin the oracle's pieces (bf16 rounding, RMSNorm, RoPE, attention)
to torch's own formulations.  ``gpu`` tests check each shell kernel against
a torch or float64 reference of the same op, and a two-layer decoder step
(packed projections + shell) against ``oracle.decoder_oracle`` with the
full-model bound: logits cosine >= 0.9999.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import decoder_oracle as do
from oracle import packed_oracle as po


def test_oracle_bf16_rounding_matches_torch() -> None:
    x = (np.random.default_rng(0).standard_normal(10000) * 10).astype(np.float32)
    x[:4] = (1.00390625, 1.01171875, -3.0e-39, 65504.0)  # ties and tiny values
    expected = torch.from_numpy(x).bfloat16().float().numpy()
    assert np.array_equal(do.bf16(x), expected)


def test_oracle_pieces_match_torch_formulas() -> None:
    rng = np.random.default_rng(1)
    x = rng.standard_normal((3, 64)).astype(np.float32)
    w = (1 + 0.02 * rng.standard_normal(64)).astype(np.float32)
    t = torch.from_numpy(x).double()
    ref = (t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-6) * torch.from_numpy(w).double()).float().numpy()
    np.testing.assert_allclose(do.rmsnorm(x, w, 1e-6), ref, rtol=1e-6, atol=1e-6)
    cos, sin = do.rope_tables(np.arange(5, 8), 64, 1e6)
    rot = do.rotate(x, cos, sin)
    # a rotation keeps the norm of every (i, i + 32) pair
    np.testing.assert_allclose(rot[:, :32] ** 2 + rot[:, 32:] ** 2, x[:, :32] ** 2 + x[:, 32:] ** 2, rtol=1e-5)
    q = rng.standard_normal((2, 4, 64)).astype(np.float32)
    kc = rng.standard_normal((2, 40, 64)).astype(np.float32)
    vc = rng.standard_normal((2, 40, 64)).astype(np.float32)
    out = do.attention(q, kc, vc, 30)
    for tok in range(2):
        for h in range(4):
            s = torch.from_numpy(kc[h // 2, : 30 + tok]).double() @ torch.from_numpy(q[tok, h]).double() / 8.0
            ref = torch.softmax(s, 0) @ torch.from_numpy(vc[h // 2, : 30 + tok]).double()
            np.testing.assert_allclose(out[tok, h], ref.numpy(), rtol=1e-5, atol=1e-6)


# ------------------------------------------------------------------ GPU ---


def _gpu() -> torch.device:
    if not torch.cuda.is_available():
        pytest.fail("GPU test needs CUDA")
    return torch.device("cuda", 0)


@pytest.mark.gpu
@pytest.mark.parametrize("delta", (False, True))
@pytest.mark.parametrize(("hidden", "w_dtype", "out_dtype"), (
    (4096, torch.bfloat16, torch.bfloat16), (4096, torch.float32, torch.float32), (1152, torch.float16, torch.float16),
    (1150, torch.bfloat16, torch.bfloat16), (12288, torch.bfloat16, torch.float32)))
def test_rmsnorm_kernel(delta: bool, hidden: int, w_dtype: torch.dtype, out_dtype: torch.dtype) -> None:
    # rows of up to 8192 values (a multiple of 4) take the register path; 1150 and 12288 the loop
    from nanoquant_b200.decoder import rmsnorm

    dev = _gpu()
    g = torch.Generator(device=dev).manual_seed(3)
    h = torch.randn(5, hidden, generator=g, device=dev)
    d = torch.randn(5, hidden, generator=g, device=dev) if delta else None
    w = (1 + 0.02 * torch.randn(hidden, generator=g, device=dev)).to(w_dtype)
    out = torch.empty(5, hidden, dtype=out_dtype, device=dev)
    ref_h = h + d if delta else h.clone()
    rmsnorm(h, d, w, 1e-6, out)
    torch.testing.assert_close(h, ref_h, rtol=0, atol=0)
    hd = ref_h.double()
    ref = (hd * torch.rsqrt(hd.pow(2).mean(-1, keepdim=True) + 1e-6) * w.double()).float()
    torch.testing.assert_close(out.float(), ref, rtol=8e-3, atol=1e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("head_dim", (64, 128, 256))
def test_qk_norm_rope_kernel(head_dim: int) -> None:
    from nanoquant_b200.decoder import qk_norm_rope, rope_tables

    dev = _gpu()
    g = torch.Generator(device=dev).manual_seed(head_dim)
    tokens, hq, hkv, pos, cache = 3, 8, 2, 11, 20
    q = torch.randn(tokens, hq * head_dim, generator=g, device=dev)
    k = torch.randn(tokens, hkv * head_dim, generator=g, device=dev)
    v = torch.randn(tokens, hkv * head_dim, generator=g, device=dev)
    qw = (1 + 0.02 * torch.randn(head_dim, generator=g, device=dev)).bfloat16()
    kw = (1 + 0.02 * torch.randn(head_dim, generator=g, device=dev)).bfloat16()
    cos, sin = (t.to(dev) for t in rope_tables(torch.arange(pos, pos + tokens), head_dim, 1e6))
    q_out = torch.empty(tokens, hq * head_dim, dtype=torch.bfloat16, device=dev)
    kc = torch.zeros(hkv, cache, head_dim, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    qk_norm_rope(q, k, v, qw, kw, cos, sin, q_out, kc, vc, pos, 1e-6, hq, hkv, head_dim)
    c, s = do.rope_tables(np.arange(pos, pos + tokens), head_dim, 1e6)
    ref_q = do.rotate(do.rmsnorm(q.cpu().numpy().reshape(tokens, hq, head_dim), qw.float().cpu().numpy(), 1e-6),
                      c[:, None], s[:, None])
    ref_k = do.rotate(do.rmsnorm(k.cpu().numpy().reshape(tokens, hkv, head_dim), kw.float().cpu().numpy(), 1e-6),
                      c[:, None], s[:, None])
    np.testing.assert_allclose(q_out.float().cpu().numpy().reshape(tokens, hq, head_dim), ref_q, rtol=8e-3, atol=8e-3)
    for t in range(tokens):
        np.testing.assert_allclose(kc[:, pos + t].float().cpu().numpy(), ref_k[t], rtol=8e-3, atol=8e-3)
        np.testing.assert_array_equal(vc[:, pos + t].float().cpu().numpy(),
                                      do.bf16(v.cpu().numpy().reshape(tokens, hkv, head_dim)[t]))
    assert not kc[:, :pos].any() and not kc[:, pos + tokens:].any()


@pytest.mark.gpu
@pytest.mark.parametrize(("head_dim", "keys", "tokens"),
                         ((64, 1, 1), (128, 300, 3), (128, 2049, 1), (128, 2049, 16), (256, 77, 16),
                          # past 4096 keys a split stages more than one 64-key load (the staged rows are reused)
                          (128, 5000, 1), (128, 9000, 16), (256, 5000, 16), (256, 9000, 1)))
def test_decode_attention_kernel(head_dim: int, keys: int, tokens: int) -> None:
    from nanoquant_b200.decoder import attention_workspace_bytes, decode_attention

    dev = _gpu()
    g = torch.Generator(device=dev).manual_seed(keys)
    hq, hkv, cache = 8, 2, keys + tokens + 5
    q = torch.randn(tokens, hq * head_dim, generator=g, device=dev).bfloat16()
    kc = torch.randn(hkv, cache, head_dim, generator=g, device=dev).bfloat16()
    vc = torch.randn(hkv, cache, head_dim, generator=g, device=dev).bfloat16()
    out = torch.empty(tokens, hq * head_dim, dtype=torch.bfloat16, device=dev)
    ws = torch.empty(attention_workspace_bytes(keys, tokens, hq, head_dim), dtype=torch.uint8, device=dev)
    decode_attention(q, kc, vc, keys, hq, hkv, head_dim, out, ws)
    ref = do.attention(q.float().cpu().numpy().reshape(tokens, hq, head_dim), kc.float().cpu().numpy(),
                       vc.float().cpu().numpy(), keys)
    np.testing.assert_allclose(out.float().cpu().numpy().reshape(tokens, hq, head_dim), ref, rtol=1e-2, atol=1e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("tokens", (1, 3, 9, 16))
def test_silu_mul_and_gemv_kernels(tokens: int) -> None:
    from nanoquant_b200.decoder import gemv_bf16, silu_mul

    dev = _gpu()
    g = torch.Generator(device=dev).manual_seed(tokens)
    gate = torch.randn(tokens, 700, generator=g, device=dev)
    up = torch.randn(tokens, 700, generator=g, device=dev)
    act = torch.empty(tokens, 700, dtype=torch.bfloat16, device=dev)
    silu_mul(gate, up, act)
    torch.testing.assert_close(act.float(), (torch.nn.functional.silu(gate) * up).bfloat16().float(), rtol=8e-3,
                               atol=8e-3)
    w = (0.02 * torch.randn(1003, 4096, generator=g, device=dev)).bfloat16()
    x = torch.randn(tokens, 4096, generator=g, device=dev).bfloat16()
    out = torch.empty(tokens, 1003, device=dev)
    gemv_bf16(w, x, out)
    ref = (x.double() @ w.double().T).float()
    torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-4)


@pytest.mark.gpu
@pytest.mark.parametrize(("tokens", "cols"), ((2, 4096), (8, 4096), (9, 4096), (16, 4096), (19, 4096), (5, 1000),
                                              (16, 2048)))
def test_gemv_tensor_core_tiles(tokens: int, cols: int) -> None:
    """2..16 tokens per launch take the mma.sync kernel (columns a multiple of 32), other widths the CUDA cores;
    more than 16 tokens run in chunks.  Rows past a 16-row tile and tokens past an 8-token tile are masked."""

    from nanoquant_b200.decoder import gemv_bf16

    dev = _gpu()
    g = torch.Generator(device=dev).manual_seed(tokens * cols)
    w = (0.02 * torch.randn(2053, cols, generator=g, device=dev)).bfloat16()
    x = torch.randn(tokens, cols, generator=g, device=dev).bfloat16()
    out = torch.full((tokens, 2053), 7.0, device=dev)
    gemv_bf16(w, x, out)
    ref = (x.double() @ w.double().T).float()
    torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-4)


def _tiny_shape():
    from nanoquant_b200.decode_chain import DecoderShape

    return DecoderShape("tiny", 2, 256, 512, 4, 2, 64, 1.0)


def _host_state(state):
    from dataclasses import fields, replace

    moved = {f.name: getattr(state, f.name).cpu() for f in fields(state)
             if isinstance(getattr(state, f.name), torch.Tensor)}
    return replace(state, **moved)


@pytest.mark.gpu
@pytest.mark.parametrize("tokens", (1, 3))
def test_decoder_step_matches_oracle(tokens: int) -> None:
    from nanoquant_b200.decode_chain import make_decoder_layers
    from nanoquant_b200.decoder import Qwen3DecodeStep, random_shell_weights
    from tests.test_cuda_parity import oracle_from_state

    dev = _gpu()
    shape = _tiny_shape()
    blocks = make_decoder_layers(shape, dev, layers=2, seed=4)
    shell = random_shell_weights(shape, 1000, dev, layers=2, seed=5)
    step = Qwen3DecodeStep(shape, blocks, shell, dev, tokens=tokens, position=37)
    k0 = [layer["k_cache"].float().cpu().numpy() for layer in step.layers]
    v0 = [layer["v_cache"].float().cpu().numpy() for layer in step.layers]
    hidden = torch.randn(tokens, shape.hidden, generator=torch.Generator(device=dev).manual_seed(6), device=dev)
    logits = step.step(hidden).cpu().numpy()
    torch.cuda.synchronize()
    layers = [{name: oracle_from_state(_host_state(state)) for name, state in block.items()} for block in blocks]
    norms = {
        "input_norm": [w.float().cpu().numpy() for w in shell.input_norm],
        "post_norm": [w.float().cpu().numpy() for w in shell.post_norm],
        "q_norm": [w.float().cpu().numpy() for w in shell.q_norm],
        "k_norm": [w.float().cpu().numpy() for w in shell.k_norm],
        "final_norm": shell.final_norm.float().cpu().numpy(),
        "lm_head": shell.lm_head.float().cpu().numpy(),
    }
    ref, k1, v1 = do.decode_step(hidden.cpu().numpy(), layers, norms, k0, v0, position=37, q_heads=4, kv_heads=2,
                                 head_dim=64, eps=1e-6, theta=1e6)
    for a, b in zip(logits, ref, strict=True):
        cosine = float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))
        assert cosine >= 0.9999, cosine
    assert float(np.abs(logits - ref).max() / np.abs(ref).max()) <= 2e-2
    for i, layer in enumerate(step.layers):
        got_v = layer["v_cache"].float().cpu().numpy()
        np.testing.assert_array_equal(got_v[:, :37], v0[i][:, :37])
        np.testing.assert_allclose(got_v[:, 37:37 + tokens], v1[i][:, 37:37 + tokens], rtol=2e-2, atol=2e-2)
        np.testing.assert_allclose(layer["k_cache"].float().cpu().numpy()[:, 37:37 + tokens],
                                   k1[i][:, 37:37 + tokens], rtol=2e-2, atol=2e-2)


@pytest.mark.gpu
@pytest.mark.parametrize(("tokens", "pos"), ((1, 300), (3, 300), (16, 300), (1, 9000), (16, 9000)))
def test_fused_decoder_step_matches_oracle(tokens: int, pos: int) -> None:
    """The fused engine (one program for every layer: residual-stream norms, q/k norm + RoPE + cache append and
    attention inside it) against the oracle with fp32 normalised activations; caches and shell path agree.

    At 9000 cached tokens each attention split holds more rows than the sign ring carries, so its last rows
    come from global memory.
    """

    from nanoquant_b200.decode_chain import DecoderShape, make_decoder_layers
    from nanoquant_b200.decoder import Qwen3DecodeStep, random_shell_weights
    from tests.test_cuda_parity import oracle_from_state

    dev = _gpu()
    shape = DecoderShape("fusable", 3, 512, 1024, 8, 2, 128, 1.0)
    blocks = make_decoder_layers(shape, dev, layers=3, seed=24)
    shell = random_shell_weights(shape, 2000, dev, layers=3, seed=25)
    step = Qwen3DecodeStep(shape, blocks, shell, dev, tokens=tokens, position=pos,
                           kv_init=torch.Generator(device=dev).manual_seed(26))
    assert step.engine == "fused" and step.kernel_launches() == 4
    k0 = [layer["k_cache"].float().cpu().numpy() for layer in step.layers]
    v0 = [layer["v_cache"].float().cpu().numpy() for layer in step.layers]
    hidden = torch.randn(tokens, shape.hidden, generator=torch.Generator(device=dev).manual_seed(27), device=dev)
    logits = step.step(hidden).cpu().numpy()
    again = step.step(hidden).cpu().numpy()
    torch.cuda.synchronize()
    assert np.array_equal(logits, again)  # deterministic
    layers = [{name: oracle_from_state(_host_state(state)) for name, state in block.items()} for block in blocks]
    norms = {
        "input_norm": [w.float().cpu().numpy() for w in shell.input_norm],
        "post_norm": [w.float().cpu().numpy() for w in shell.post_norm],
        "q_norm": [w.float().cpu().numpy() for w in shell.q_norm],
        "k_norm": [w.float().cpu().numpy() for w in shell.k_norm],
        "final_norm": shell.final_norm.float().cpu().numpy(),
        "lm_head": shell.lm_head.float().cpu().numpy(),
    }
    ref, k1, v1 = do.decode_step(hidden.cpu().numpy(), layers, norms, k0, v0, position=pos, q_heads=8, kv_heads=2,
                                 head_dim=128, eps=1e-6, theta=1e6, xn_bf16=False)
    for a, b in zip(logits, ref, strict=True):
        cosine = float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))
        assert cosine >= 0.99999, cosine
    for i, layer in enumerate(step.layers):
        np.testing.assert_allclose(layer["k_cache"].float().cpu().numpy()[:, pos:pos + tokens],
                                   k1[i][:, pos:pos + tokens], rtol=2e-2, atol=2e-2)
        np.testing.assert_allclose(layer["v_cache"].float().cpu().numpy()[:, pos:pos + tokens],
                                   v1[i][:, pos:pos + tokens], rtol=2e-2, atol=2e-2)
        assert np.array_equal(layer["k_cache"].float().cpu().numpy()[:, :pos], k0[i][:, :pos])


@pytest.mark.gpu
def test_decoder_step_graph_replay_is_bitwise_eager() -> None:
    from nanoquant_b200.decoder import build_qwen3_step

    dev = _gpu()
    step = build_qwen3_step(_tiny_shape(), dev, vocab=512, tokens=2, position=9, layers=2, seed=7)
    hidden = torch.randn(2, 256, generator=torch.Generator(device=dev).manual_seed(8), device=dev)
    eager = step.step(hidden).clone()
    step.capture()
    first = step.replay().clone()
    second = step.replay().clone()
    torch.cuda.synchronize()
    assert torch.equal(eager, first) and torch.equal(first, second)


def test_oracle_independent_sequences_match_single_token_steps() -> None:
    """The oracle's batch of independent sequences equals one single-token step per sequence (CPU)."""

    rng = np.random.default_rng(40)
    tokens, hidden, q_heads, kv_heads, hd, position = 3, 64, 4, 1, 32, 5

    def layer(n: int, m: int) -> po.OracleLayer:
        r = 16
        left = rng.integers(0, 2**16, size=(m, 1), dtype=np.int64).astype(np.int32)
        right = rng.integers(0, 2**31, size=(r, (n + 31) // 32), dtype=np.int64).astype(np.int32)
        return po.OracleLayer(n, m, r, left, right, np.full(n, 0.05, np.float32), np.ones(r, np.float32),
                              np.full(m, 0.05, np.float32))

    proj = {"q_proj": layer(hidden, q_heads * hd), "k_proj": layer(hidden, kv_heads * hd),
            "v_proj": layer(hidden, kv_heads * hd), "o_proj": layer(q_heads * hd, hidden),
            "gate_proj": layer(hidden, 96), "up_proj": layer(hidden, 96), "down_proj": layer(96, hidden)}
    norms = {"input_norm": [np.ones(hidden, np.float32)], "post_norm": [np.ones(hidden, np.float32)],
             "q_norm": [np.ones(hd, np.float32)], "k_norm": [np.ones(hd, np.float32)],
             "final_norm": np.ones(hidden, np.float32), "lm_head": rng.standard_normal((50, hidden)).astype(np.float32)}
    hidden_in = rng.standard_normal((tokens, hidden)).astype(np.float32)
    k = do.bf16(rng.standard_normal((tokens, kv_heads, position + 1, hd)).astype(np.float32))
    v = do.bf16(rng.standard_normal((tokens, kv_heads, position + 1, hd)).astype(np.float32))
    batch, kb, vb = do.decode_step(hidden_in, [proj], norms, [k], [v], position=position, q_heads=q_heads,
                                   kv_heads=kv_heads, head_dim=hd, eps=1e-6, theta=1e6, sequences=True)
    for t in range(tokens):
        one, k1, v1 = do.decode_step(hidden_in[t:t + 1], [proj], norms, [k[t]], [v[t]], position=position,
                                     q_heads=q_heads, kv_heads=kv_heads, head_dim=hd, eps=1e-6, theta=1e6)
        np.testing.assert_allclose(batch[t], one[0], rtol=1e-5, atol=1e-6)
        np.testing.assert_array_equal(kb[0][t], k1[0])
        np.testing.assert_array_equal(vb[0][t], v1[0])


@pytest.mark.gpu
@pytest.mark.parametrize(("tokens", "pos"), ((2, 300), (16, 300), (16, 9000)))
def test_fused_step_over_independent_sequences_matches_oracle(tokens: int, pos: int) -> None:
    """A batch of independent sequences (own caches per token, all at one position) in the fused program."""

    from nanoquant_b200.decode_chain import DecoderShape, make_decoder_layers
    from nanoquant_b200.decoder import Qwen3DecodeStep, random_shell_weights
    from tests.test_cuda_parity import oracle_from_state

    dev = _gpu()
    shape = DecoderShape("fusable", 2, 512, 1024, 8, 2, 128, 1.0)
    blocks = make_decoder_layers(shape, dev, layers=2, seed=44)
    shell = random_shell_weights(shape, 2000, dev, layers=2, seed=45)
    step = Qwen3DecodeStep(shape, blocks, shell, dev, tokens=tokens, position=pos, sequences=True,
                           kv_init=torch.Generator(device=dev).manual_seed(46))
    assert step.layers[0]["k_cache"].shape == (tokens, 2, pos + 1, 128)
    k0 = [layer["k_cache"].float().cpu().numpy() for layer in step.layers]
    v0 = [layer["v_cache"].float().cpu().numpy() for layer in step.layers]
    hidden = torch.randn(tokens, shape.hidden, generator=torch.Generator(device=dev).manual_seed(47), device=dev)
    logits = step.step(hidden).cpu().numpy()
    again = step.step(hidden).cpu().numpy()
    torch.cuda.synchronize()
    assert np.array_equal(logits, again)
    layers = [{name: oracle_from_state(_host_state(state)) for name, state in block.items()} for block in blocks]
    norms = {
        "input_norm": [w.float().cpu().numpy() for w in shell.input_norm],
        "post_norm": [w.float().cpu().numpy() for w in shell.post_norm],
        "q_norm": [w.float().cpu().numpy() for w in shell.q_norm],
        "k_norm": [w.float().cpu().numpy() for w in shell.k_norm],
        "final_norm": shell.final_norm.float().cpu().numpy(),
        "lm_head": shell.lm_head.float().cpu().numpy(),
    }
    ref, k1, v1 = do.decode_step(hidden.cpu().numpy(), layers, norms, k0, v0, position=pos, q_heads=8, kv_heads=2,
                                 head_dim=128, eps=1e-6, theta=1e6, xn_bf16=False, sequences=True)
    for a, b in zip(logits, ref, strict=True):
        cosine = float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))
        assert cosine >= 0.99999, cosine
    for i, layer in enumerate(step.layers):
        kc, vc = layer["k_cache"].float().cpu().numpy(), layer["v_cache"].float().cpu().numpy()
        np.testing.assert_allclose(kc[:, :, pos], k1[i][:, :, pos], rtol=2e-2, atol=2e-2)
        np.testing.assert_allclose(vc[:, :, pos], v1[i][:, :, pos], rtol=2e-2, atol=2e-2)
        assert np.array_equal(kc[:, :, :pos], k0[i][:, :, :pos])


@pytest.mark.gpu
def test_program_rejects_sequence_caches_too_short() -> None:
    """With independent sequences each cache must hold row ``position``: the host refuses the program otherwise."""

    from nanoquant_b200 import _native
    from nanoquant_b200.decode_chain import DecoderShape, make_decoder_layers
    from nanoquant_b200.decoder import Qwen3DecodeStep, random_shell_weights

    dev = _gpu()
    shape = DecoderShape("fusable", 1, 512, 1024, 8, 2, 128, 1.0)
    blocks = make_decoder_layers(shape, dev, layers=1, seed=48)
    shell = random_shell_weights(shape, 500, dev, layers=1, seed=49)
    step = Qwen3DecodeStep(shape, blocks, shell, dev, tokens=2, position=64, sequences=True)
    step.cache_len = 64  # rows [0, 64) only: the new row 64 does not fit
    with pytest.raises(_native.NativeError) as err:
        step._fused_program()
    assert err.value.status == _native.NQB_ERR_INVALID_ARGUMENT
