"""A Qwen3-style decoder step around the packed linears (batch 1..16).

The decode-step shell: what a decoder layer does besides its seven packed
projections.  Per layer

    xn   = rmsnorm(h) * w_in                       (bf16)
    q, k, v = qkv(xn)                              (one persistent program)
    q, k = rope(rmsnorm_head(q) * q_norm), rope(rmsnorm_head(k) * k_norm)
    cache[pos + t] <- k, v                         (bf16 caches)
    a    = attention(q, cache)                     (grouped-query, split-K)
    h   += o_proj(a);   xn2 = rmsnorm(h) * w_post
    h   += down(silu(gate(xn2)) * up(xn2))

then ``logits = lm_head(rmsnorm(h) * w_final)`` with a dense bf16 lm head.
The shell kernels are ``nqb_rmsnorm``, ``nqb_qk_norm_rope``,
``nqb_decode_attention``, ``nqb_silu_mul`` and ``nqb_gemv_bf16``; the packed
projections run as three decode programs per layer: qkv, o, and an MLP
program whose second op forms ``silu(gate) * up`` as it loads its input (so
``nqb_silu_mul`` runs only for a down projection with salient columns, which
the fused input does not take).  This mirrors the
reference's model shell (``src/nanoquant/runtime/torch_model.py:185-421``),
which runs the same math with torch modules and Triton kernels pinned to one
geometry (``cuda_kernels.py:401-812``).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from nanoquant_b200 import _native
from nanoquant_b200.cuda_backend import CudaPackedSm100Backend
from nanoquant_b200.decode_chain import DecoderShape, make_decoder_layers
from nanoquant_b200.program import DecodeProgram, ProgramOp


def _stream(device: torch.device) -> int:
    return _native.current_stream_handle(device)


def rmsnorm(h: torch.Tensor, delta: torch.Tensor | None, weight: torch.Tensor, eps: float, out: torch.Tensor,
            delta_weight: torch.Tensor | None = None) -> None:
    """``h += delta`` (when given), ``out = h * rsqrt(mean(h^2) + eps) * weight`` per token (``nqb_rmsnorm``).

    With ``delta_weight`` the delta is RMS-normalised with it before the add
    (``nqb_rmsnorm_residual``: Gemma-3's post-attention / post-feedforward norms).
    """

    tokens, hidden = h.shape
    if delta_weight is not None and delta_weight.dtype != weight.dtype:
        raise ValueError("both norm weights share one dtype")
    _native.call("nqb_rmsnorm_residual", h.data_ptr(), 0 if delta is None else delta.data_ptr(),
                 0 if delta_weight is None else delta_weight.data_ptr(), weight.data_ptr(),
                 _native.dtype_code(weight.dtype), tokens, hidden, ctypes.c_float(eps), out.data_ptr(),
                 _native.dtype_code(out.dtype), _stream(h.device))


def qk_norm_rope(q, k, v, q_weight, k_weight, cos, sin, q_out, k_cache, v_cache, position: int, eps: float,
                 q_heads: int, kv_heads: int, head_dim: int) -> None:
    """Per-head q/k RMSNorm and rotate-half RoPE; k, v appended to the caches (``nqb_qk_norm_rope``)."""

    tokens = q.shape[0]
    _native.call("nqb_qk_norm_rope", q.data_ptr(), k.data_ptr(), v.data_ptr(),
                 0 if q_weight is None else q_weight.data_ptr(), 0 if k_weight is None else k_weight.data_ptr(),
                 _native.dtype_code(q_weight.dtype if q_weight is not None else torch.float32), cos.data_ptr(),
                 sin.data_ptr(), tokens, q_heads, kv_heads, head_dim, ctypes.c_float(eps), q_out.data_ptr(),
                 k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[1], position, _stream(q.device))


def attention_workspace_bytes(keys: int, tokens: int, q_heads: int, head_dim: int) -> int:
    size = ctypes.c_size_t(0)
    _native.call("nqb_decode_attention_workspace_bytes", keys, tokens, q_heads, head_dim, ctypes.byref(size))
    return size.value


def decode_attention(q, k_cache, v_cache, keys: int, q_heads: int, kv_heads: int, head_dim: int, out,
                     workspace: torch.Tensor, window: int = 0) -> None:
    """Grouped-query attention of ``tokens`` queries over the caches (``nqb_decode_attention_window``).

    ``window > 0``: token t sees only the last ``window`` cache rows ending at its own.
    """

    _native.call("nqb_decode_attention_window", q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                 k_cache.shape[1], keys, q.shape[0], q_heads, kv_heads, head_dim, window, out.data_ptr(),
                 workspace.data_ptr(), workspace.numel(), _stream(q.device))


def embedding_bf16(ids: torch.Tensor, weight: torch.Tensor, scale: float, out: torch.Tensor) -> None:
    """``out[t] = weight[ids[t]] * scale`` in fp32 (``nqb_embedding_bf16``)."""

    _native.call("nqb_embedding_bf16", ids.data_ptr(), ids.numel(), weight.data_ptr(), weight.shape[0],
                 weight.shape[1], ctypes.c_float(scale), out.data_ptr(), _stream(ids.device))


def silu_mul(gate: torch.Tensor, up: torch.Tensor, out: torch.Tensor) -> None:
    """``out = silu(gate) * up`` (``nqb_silu_mul``)."""

    _native.call("nqb_silu_mul", gate.data_ptr(), up.data_ptr(), gate.numel(), out.data_ptr(),
                 _native.dtype_code(out.dtype), _stream(gate.device))


def gemv_bf16(weight: torch.Tensor, x: torch.Tensor, out: torch.Tensor) -> None:
    """``out[t] = weight @ x[t]`` with a bf16 ``weight`` streamed once (``nqb_gemv_bf16``)."""

    _native.call("nqb_gemv_bf16", weight.data_ptr(), weight.shape[0], weight.shape[1], x.data_ptr(), x.shape[0],
                 out.data_ptr(), _stream(x.device))


def rope_tables(positions: torch.Tensor, head_dim: int, theta: float) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin rows ``[len(positions), head_dim]`` (halves duplicated), fp32."""

    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    angles = positions.to(torch.float64)[:, None] * inv[None, :]
    emb = torch.cat((angles, angles), dim=-1)
    return emb.cos().float(), emb.sin().float()


@dataclass
class ShellWeights:
    """The dense (non-packed) weights of one decoder: per-layer norms, final norm, lm head."""

    input_norm: list[torch.Tensor]
    post_norm: list[torch.Tensor]
    q_norm: list[torch.Tensor]
    k_norm: list[torch.Tensor]
    final_norm: torch.Tensor
    lm_head: torch.Tensor


def random_shell_weights(shape: DecoderShape, vocab: int, device: torch.device, *, layers: int | None = None,
                         seed: int = 1) -> ShellWeights:
    """bf16 norms ``1 + N(0, 0.02)`` and a bf16 lm head ``N(0, 0.02)`` (random init)."""

    g = torch.Generator(device=device).manual_seed(seed)
    count = shape.layers if layers is None else layers

    def norm(size: int) -> torch.Tensor:
        return (1.0 + 0.02 * torch.randn(size, generator=g, device=device)).bfloat16()

    return ShellWeights(
        [norm(shape.hidden) for _ in range(count)], [norm(shape.hidden) for _ in range(count)],
        [norm(shape.head_dim) for _ in range(count)], [norm(shape.head_dim) for _ in range(count)],
        norm(shape.hidden), (0.02 * torch.randn(vocab, shape.hidden, generator=g, device=device)).bfloat16())


def residual_stats(h: torch.Tensor, stats: torch.Tensor) -> None:
    """Per-128-row sums of squares of the residual stream ``h [T, hidden]`` into ``stats`` (``nqb_residual_stats``)."""

    _native.call("nqb_residual_stats", h.data_ptr(), h.shape[0], h.shape[1], stats.data_ptr(), _stream(h.device))


class Qwen3DecodeStep:
    """One decode step of ``tokens`` new tokens at cache position ``position``.

    ``blocks``: per layer the packed states of q/k/v/o/gate/up/down (as from
    :func:`make_decoder_layers`); ``shell``: the dense weights; the KV caches
    hold ``position`` prior tokens (rows ``[0, position)``, random N(0, 1)
    here) and get the new tokens' keys and values at rows ``position + t``.
    :meth:`step` returns the fp32 logits ``[tokens, vocab]``; the position
    does not advance (each step recomputes the same tokens), so replays of a
    captured step are identical.

    ``engine="fused"`` (default; head_dim 128, 4 q heads per kv head): every
    layer runs inside ONE persistent program -- per layer a q/k/v op that
    normalises the residual stream as it loads it and ends in the q/k norm,
    RoPE and cache append, the attention op, o with the residual add, gate/up
    with the post-attention norm folded in, and down (SwiGLU input) with the
    residual add -- then the final norm and the lm head: four launches per
    step.  The normalised activations stay fp32 (no bf16 rounding).
    ``engine="shell"``: three programs per layer around separate shell kernels
    (norms, q/k norm + RoPE, attention), with bf16 normalised activations.

    ``sequences=True`` (fused engine): the tokens are a batch of independent
    sequences instead, token t the next token of sequence t with its own
    caches (``k_cache[t]`` / ``v_cache[t]``, each ``[kv_heads, cache_len,
    head_dim]``, ``position`` prior rows), all at position ``position``.
    """

    def __init__(self, shape: DecoderShape, blocks, shell: ShellWeights, device: torch.device, *, tokens: int = 1,
                 position: int = 0, cache_len: int | None = None, eps: float = 1e-6, rope_theta: float = 1e6,
                 kv_init: torch.Generator | None = None, engine: str | None = None, sequences: bool = False) -> None:
        if not 1 <= tokens <= 16:
            raise ValueError("a decode step takes 1 to 16 tokens")
        fusable = shape.head_dim == 128 and shape.q_heads == 4 * shape.kv_heads
        engine = engine or ("fused" if fusable else "shell")
        if engine not in ("fused", "shell") or (engine == "fused" and not fusable):
            raise ValueError(f"engine {engine!r} is not available for this shape")
        if sequences and engine != "fused":
            raise ValueError("independent sequences run on the fused engine only")
        self.engine = engine
        self.sequences = sequences
        self.shape, self.device, self.tokens, self.position, self.eps = shape, device, tokens, position, eps
        self.shell = shell
        new_rows = 1 if sequences else tokens
        self.cache_len = cache_len if cache_len is not None else position + new_rows
        if position + new_rows > self.cache_len:
            raise ValueError("the cache is too short for the step's tokens")
        backend = CudaPackedSm100Backend()
        hd, hq, hkv = shape.head_dim, shape.q_heads, shape.kv_heads
        f32 = {"dtype": torch.float32, "device": device}
        bf16 = {"dtype": torch.bfloat16, "device": device}
        self.hidden_in = torch.zeros(tokens, shape.hidden, **f32)  # the step's input embeddings
        self.h = torch.zeros(tokens, shape.hidden, **f32)  # residual stream
        self.xn = torch.zeros(tokens, shape.hidden, **bf16)
        self.q_rot = torch.zeros(tokens, hq * hd, **bf16)
        self.attn = torch.zeros(tokens, hq * hd, **bf16)
        self.act = torch.zeros(tokens, shape.intermediate, **bf16)
        self.logits = torch.zeros(tokens, shell.lm_head.shape[0], **f32)
        self.keys = position + 1
        self.attn_ws = torch.empty(attention_workspace_bytes(self.keys, tokens, hq, hd), dtype=torch.uint8,
                                   device=device)
        positions = torch.full((tokens,), position) if sequences else torch.arange(position, position + tokens)
        self.cos, self.sin = (t.to(device) for t in rope_tables(positions, hd, rope_theta))
        g = kv_init if kv_init is not None else torch.Generator(device=device).manual_seed(2)
        self.layers = []
        for block in blocks:
            prepared = {name: backend.prepare(state, device) for name, state in block.items()}
            q = torch.zeros(tokens, hq * hd, **f32)
            k = torch.zeros(tokens, hkv * hd, **f32)
            v = torch.zeros(tokens, hkv * hd, **f32)
            o = torch.zeros(tokens, shape.hidden, **f32)
            gate = torch.zeros(tokens, shape.intermediate, **f32)
            up = torch.zeros(tokens, shape.intermediate, **f32)
            down = torch.zeros(tokens, shape.hidden, **f32)
            lead = (tokens,) if sequences else ()
            kc = torch.zeros(*lead, hkv, self.cache_len, hd, **bf16)
            vc = torch.zeros(*lead, hkv, self.cache_len, hd, **bf16)
            if position:
                kc[..., :position, :] = torch.randn(*lead, hkv, position, hd, generator=g, device=device).bfloat16()
                vc[..., :position, :] = torch.randn(*lead, hkv, position, hd, generator=g, device=device).bfloat16()
            layer = {"q": q, "k": k, "v": v, "o": o, "gate": gate, "up": up, "down": down, "k_cache": kc,
                     "v_cache": vc, "prepared": prepared}
            if engine == "shell":
                layer.update({
                    "prog_qkv": DecodeProgram([ProgramOp((prepared["q_proj"], prepared["k_proj"],
                                                          prepared["v_proj"]), self.xn)], outputs=[(q, k, v)]),
                    "prog_o": DecodeProgram([ProgramOp((prepared["o_proj"],), self.attn)], outputs=[(o,)]),
                    "prog_mlp": self._mlp_program(prepared, gate, up, down),
                })
            self.layers.append(layer)
        self.program: DecodeProgram | None = None
        if engine == "fused":
            self.stats = torch.zeros((shape.hidden + 127) // 128, tokens, **f32)
            self.program = self._fused_program()
        self.graph: torch.cuda.CUDAGraph | None = None

    def _fused_program(self) -> DecodeProgram:
        """Every layer as five ops of one program (q/k/v, attention, o, gate/up, down)."""

        s = self.shape
        ops, outputs = [], []
        w_dtype = _native.dtype_code(self.shell.input_norm[0].dtype)

        def ext(**fields) -> _native.ProgramOpExt:
            e = _native.ProgramOpExt()
            e.kind = _native.NQB_OP_LINEAR
            e.epilogue = _native.NQB_EPI_STORE
            e.eps = self.eps
            for name, value in fields.items():
                setattr(e, name, value)
            return e

        for index, layer in enumerate(self.layers):
            prepared = layer["prepared"]
            cache = {"q": self.q_rot.data_ptr(), "k_cache": layer["k_cache"].data_ptr(),
                     "v_cache": layer["v_cache"].data_ptr(), "cache_len": self.cache_len, "position": self.position,
                     "q_heads": s.q_heads, "kv_heads": s.kv_heads, "head_dim": s.head_dim,
                     "sequence_stride": s.kv_heads * self.cache_len * s.head_dim if self.sequences else 0}
            ops.append(ProgramOp((prepared["q_proj"], prepared["k_proj"], prepared["v_proj"]), self.h, ext=ext(
                epilogue=_native.NQB_EPI_QK_ROPE, norm_stats=self.stats.data_ptr(),
                norm_weight=self.shell.input_norm[index].data_ptr(), norm_weight_dtype=w_dtype,
                q_norm_weight=self.shell.q_norm[index].data_ptr(), k_norm_weight=self.shell.k_norm[index].data_ptr(),
                qk_norm_dtype=_native.dtype_code(self.shell.q_norm[index].dtype), cos_table=self.cos.data_ptr(),
                sin_table=self.sin.data_ptr(), **cache)))
            outputs.append((layer["q"], layer["k"], layer["v"]))  # not written: the epilogue stores q and the caches
            ops.append(ProgramOp((), None, ext=ext(kind=_native.NQB_OP_ATTENTION, attn_out=self.attn.data_ptr(),
                                                   **cache)))
            outputs.append(())
            ops.append(ProgramOp((prepared["o_proj"],), self.attn, ext=ext(
                epilogue=_native.NQB_EPI_RESIDUAL, out_stats=self.stats.data_ptr())))
            outputs.append((self.h,))
            ops.append(ProgramOp((prepared["gate_proj"], prepared["up_proj"]), self.h, ext=ext(
                norm_stats=self.stats.data_ptr(), norm_weight=self.shell.post_norm[index].data_ptr(),
                norm_weight_dtype=w_dtype)))
            outputs.append((layer["gate"], layer["up"]))
            ops.append(ProgramOp((prepared["down_proj"],), layer["gate"], x2=layer["up"], ext=ext(
                epilogue=_native.NQB_EPI_RESIDUAL, out_stats=self.stats.data_ptr())))
            outputs.append((self.h,))
        return DecodeProgram(ops, outputs=outputs)

    def _mlp_program(self, prepared: dict, gate: torch.Tensor, up: torch.Tensor,
                     down: torch.Tensor) -> DecodeProgram | tuple[DecodeProgram, DecodeProgram]:
        """gate/up then down in one program with the SwiGLU product formed as the down op loads it; a down
        projection with salient columns or overlay rows keeps two programs around ``nqb_silu_mul``."""

        gate_up = ProgramOp((prepared["gate_proj"], prepared["up_proj"]), self.xn)
        desc = prepared["down_proj"].payload.desc
        if desc.outlier_count == 0 and desc.overlay_rows == 0:
            return DecodeProgram([gate_up, ProgramOp((prepared["down_proj"],), gate, x2=up)],
                                 outputs=[(gate, up), (down,)])
        return (DecodeProgram([gate_up], outputs=[(gate, up)]),
                DecodeProgram([ProgramOp((prepared["down_proj"],), self.act)], outputs=[(down,)]))

    def kernel_launches(self) -> int:
        """Kernels one step launches.  Fused: the residual statistics, the program, the final norm and the lm head.
        Shell: per layer 3 programs (4 with a split MLP, plus its SwiGLU kernel), 2 norms, rope and attention (2);
        then the final norm and the lm head (the input copy is a library copy)."""

        if self.engine == "fused":
            return 4
        split = sum(isinstance(layer["prog_mlp"], tuple) for layer in self.layers)
        return len(self.layers) * 8 + 2 * split + 2

    def step(self, hidden: torch.Tensor | None = None) -> torch.Tensor:
        """Run the step on the current stream from ``hidden`` (the new tokens' embeddings; default: the
        last ones given)."""

        s, hd = self.shape, self.shape.head_dim
        if hidden is not None:
            self.hidden_in.copy_(hidden)
        self.h.copy_(self.hidden_in)
        if self.program is not None:
            residual_stats(self.h, self.stats)
            self.program.run(dependent=True)
            rmsnorm(self.h, None, self.shell.final_norm, self.eps, self.xn)
            gemv_bf16(self.shell.lm_head, self.xn, self.logits)
            return self.logits
        delta = None
        for index, layer in enumerate(self.layers):
            rmsnorm(self.h, delta, self.shell.input_norm[index], self.eps, self.xn)
            layer["prog_qkv"].run(dependent=True)
            qk_norm_rope(layer["q"], layer["k"], layer["v"], self.shell.q_norm[index], self.shell.k_norm[index],
                         self.cos, self.sin, self.q_rot, layer["k_cache"], layer["v_cache"], self.position, self.eps,
                         s.q_heads, s.kv_heads, hd)
            decode_attention(self.q_rot, layer["k_cache"], layer["v_cache"], self.keys, s.q_heads, s.kv_heads, hd,
                             self.attn, self.attn_ws)
            layer["prog_o"].run(dependent=True)
            rmsnorm(self.h, layer["o"], self.shell.post_norm[index], self.eps, self.xn)
            mlp = layer["prog_mlp"]
            if isinstance(mlp, tuple):
                mlp[0].run(dependent=True)
                silu_mul(layer["gate"], layer["up"], self.act)
                mlp[1].run(dependent=True)
            else:
                mlp.run(dependent=True)
            delta = layer["down"]
        rmsnorm(self.h, delta, self.shell.final_norm, self.eps, self.xn)
        gemv_bf16(self.shell.lm_head, self.xn, self.logits)
        return self.logits

    def capture(self) -> None:
        """Record one step (from the current input) into a CUDA graph; :meth:`replay` then reruns it."""

        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self.step()
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self.step()
        self.graph = graph

    def replay(self) -> torch.Tensor:
        if self.graph is None:
            raise RuntimeError("capture() first")
        self.graph.replay()
        return self.logits

    def program_bytes(self) -> int:
        """Bytes the fused program must move: everything of the step but the final norm and the lm head."""

        return self.algorithmic_bytes() - self.shell.lm_head.numel() * 2 - self.shape.hidden * 2

    def algorithmic_bytes(self) -> int:
        """Bytes one step must move: packed weights and scales, KV rows read, lm head, norms."""

        s = self.shape
        packed = 0
        for layer in self.layers:
            for prepared in layer["prepared"].values():
                spec = prepared.spec
                packed += (spec.out_features * ((spec.rank + 31) // 32) + spec.rank * ((spec.in_features + 31) // 32)) * 4
                packed += (spec.in_features + spec.rank + spec.out_features) * 2
        rows = self.tokens * self.keys if self.sequences else self.keys + self.tokens - 1  # KV rows attention reads
        kv = len(self.layers) * 2 * s.kv_heads * rows * s.head_dim * 2
        head = self.shell.lm_head.numel() * 2
        norms = len(self.layers) * (2 * s.hidden + 2 * s.head_dim) * 2 + s.hidden * 2
        return packed + kv + head + norms


@dataclass
class GemmaShellWeights:
    """The dense weights of a Gemma-3 decoder: per-layer norms (stored weights w, applied as 1 + w), the final
    norm and the bf16 embedding table."""

    input_norm: list[torch.Tensor]
    post_attention_norm: list[torch.Tensor]
    pre_feedforward_norm: list[torch.Tensor]
    post_feedforward_norm: list[torch.Tensor]
    q_norm: list[torch.Tensor]
    k_norm: list[torch.Tensor]
    final_norm: torch.Tensor
    embedding: torch.Tensor


def random_gemma_shell_weights(shape: DecoderShape, vocab: int, device: torch.device, *, layers: int | None = None,
                               seed: int = 1) -> GemmaShellWeights:
    """bf16 norm weights ``1 + N(0, 0.02)`` and a bf16 embedding table ``N(0, 1)`` (random init)."""

    g = torch.Generator(device=device).manual_seed(seed)
    count = shape.layers if layers is None else layers

    def norm(size: int) -> torch.Tensor:
        return (1.0 + 0.02 * torch.randn(size, generator=g, device=device)).bfloat16()

    def per_layer(size: int) -> list[torch.Tensor]:
        return [norm(size) for _ in range(count)]

    return GemmaShellWeights(per_layer(shape.hidden), per_layer(shape.hidden), per_layer(shape.hidden),
                             per_layer(shape.hidden), per_layer(shape.head_dim), per_layer(shape.head_dim),
                             norm(shape.hidden), torch.randn(vocab, shape.hidden, generator=g, device=device).bfloat16())


class Gemma3DecodeStep:
    """One Gemma-3 decode step of ``tokens`` new tokens at cache position ``position``.

    Per layer (reference ``runtime/torch_model.py:233-681``, HF Gemma-3
    semantics): ``xn = rmsnorm(h) * (1 + w_in)``; q, k, v (one program); q/k
    head norms ``(1 + w)`` and rotate-half RoPE (local layers theta 1e4 with a
    ``sliding_window``-key window, every ``global_every``-th layer global with
    theta 1e6 and full attention); attention scaled by ``head_dim^-1/2``
    (``query_pre_attn_scalar`` = head_dim); o; ``h += rmsnorm(o) * (1 +
    w_post_attn)``; ``xn = rmsnorm(h) * (1 + w_pre_ff)``; the gated-GELU MLP
    (gate/up and down with ``gelu_tanh(gate) * up`` formed as down loads it,
    one program); ``h += rmsnorm(down) * (1 + w_post_ff)``.  The sandwich
    norms run as ``nqb_rmsnorm_residual`` with the next pre-norm fused in.  The
    step starts from token ids (``nqb_embedding_bf16``, scale ``sqrt(hidden)``
    rounded to bf16 as Gemma's normaliser is) and returns the final-normed
    hidden states ``[tokens, hidden]`` fp32 (config 1 has no vocabulary head).
    Activations fed to the packed projections are fp32, like the reference's
    fp32 decode path; q, the caches and the attention output are bf16.
    """

    def __init__(self, shape: DecoderShape, blocks, shell: GemmaShellWeights, device: torch.device, *,
                 tokens: int = 1, position: int = 0, cache_len: int | None = None, eps: float = 1e-6,
                 sliding_window: int = 512, global_every: int = 6, local_theta: float = 1e4,
                 global_theta: float = 1e6, kv_init: torch.Generator | None = None) -> None:
        if not 1 <= tokens <= 16:
            raise ValueError("a decode step takes 1 to 16 tokens")
        self.shape, self.device, self.tokens, self.position, self.eps = shape, device, tokens, position, eps
        self.shell = shell
        self.cache_len = cache_len if cache_len is not None else position + tokens
        if position + tokens > self.cache_len:
            raise ValueError("the cache is too short for the step's tokens")
        backend = CudaPackedSm100Backend()
        hd, hq, hkv = shape.head_dim, shape.q_heads, shape.kv_heads
        f32 = {"dtype": torch.float32, "device": device}
        bf16 = {"dtype": torch.bfloat16, "device": device}

        def gemma(w: torch.Tensor) -> torch.Tensor:  # Gemma's RMSNorm applies (1 + w), computed in fp32
            return (1.0 + w.float()).contiguous()

        self.w_in = [gemma(w) for w in shell.input_norm]
        self.w_post_attn = [gemma(w) for w in shell.post_attention_norm]
        self.w_pre_ff = [gemma(w) for w in shell.pre_feedforward_norm]
        self.w_post_ff = [gemma(w) for w in shell.post_feedforward_norm]
        self.w_q = [gemma(w) for w in shell.q_norm]
        self.w_k = [gemma(w) for w in shell.k_norm]
        self.w_final = gemma(shell.final_norm)
        self.embed_scale = float(torch.tensor(shape.hidden ** 0.5).bfloat16().float())
        self.ids = torch.zeros(tokens, dtype=torch.int64, device=device)  # the step's input token ids
        self.h = torch.zeros(tokens, shape.hidden, **f32)
        self.xn = torch.zeros(tokens, shape.hidden, **f32)
        self.out = torch.zeros(tokens, shape.hidden, **f32)
        self.q_rot = torch.zeros(tokens, hq * hd, **bf16)
        self.attn = torch.zeros(tokens, hq * hd, **bf16)
        self.keys = position + 1
        self.attn_ws = torch.empty(attention_workspace_bytes(self.keys, tokens, hq, hd), dtype=torch.uint8,
                                   device=device)
        positions = torch.arange(position, position + tokens)
        self.rope = {theta: tuple(t.to(device) for t in rope_tables(positions, hd, theta))
                     for theta in (local_theta, global_theta)}
        g = kv_init if kv_init is not None else torch.Generator(device=device).manual_seed(2)
        self.layers = []
        for index, block in enumerate(blocks):
            prepared = {name: backend.prepare(state, device) for name, state in block.items()}
            q = torch.zeros(tokens, hq * hd, **f32)
            k = torch.zeros(tokens, hkv * hd, **f32)
            v = torch.zeros(tokens, hkv * hd, **f32)
            o = torch.zeros(tokens, shape.hidden, **f32)
            gate = torch.zeros(tokens, shape.intermediate, **f32)
            up = torch.zeros(tokens, shape.intermediate, **f32)
            down = torch.zeros(tokens, shape.hidden, **f32)
            kc = torch.zeros(hkv, self.cache_len, hd, **bf16)
            vc = torch.zeros(hkv, self.cache_len, hd, **bf16)
            if position:
                kc[:, :position] = torch.randn(hkv, position, hd, generator=g, device=device).bfloat16()
                vc[:, :position] = torch.randn(hkv, position, hd, generator=g, device=device).bfloat16()
            is_global = (index + 1) % global_every == 0
            self.layers.append({
                "prog_qkv": DecodeProgram([ProgramOp((prepared["q_proj"], prepared["k_proj"], prepared["v_proj"]),
                                                     self.xn)], outputs=[(q, k, v)]),
                "prog_o": DecodeProgram([ProgramOp((prepared["o_proj"],), self.attn)], outputs=[(o,)]),
                "prog_mlp": DecodeProgram([ProgramOp((prepared["gate_proj"], prepared["up_proj"]), self.xn),
                                           ProgramOp((prepared["down_proj"],), gate, x2=up, activation="gelu_tanh")],
                                          outputs=[(gate, up), (down,)]),
                "q": q, "k": k, "v": v, "o": o, "gate": gate, "up": up, "down": down, "k_cache": kc, "v_cache": vc,
                "prepared": prepared, "window": 0 if is_global else sliding_window,
                "theta": global_theta if is_global else local_theta,
            })
        self.graph: torch.cuda.CUDAGraph | None = None

    def kernel_launches(self) -> int:
        """Kernels one step launches: the embedding and the first norm, then per layer 3 programs, rope,
        attention (2) and 2 norms."""

        return 2 + 8 * len(self.layers)

    def step(self, ids: torch.Tensor | None = None) -> torch.Tensor:
        s, hd = self.shape, self.shape.head_dim
        if ids is not None:
            self.ids.copy_(ids)
        embedding_bf16(self.ids, self.shell.embedding, self.embed_scale, self.h)
        rmsnorm(self.h, None, self.w_in[0], self.eps, self.xn)
        last = len(self.layers) - 1
        for index, layer in enumerate(self.layers):
            cos, sin = self.rope[layer["theta"]]
            layer["prog_qkv"].run(dependent=True)
            qk_norm_rope(layer["q"], layer["k"], layer["v"], self.w_q[index], self.w_k[index], cos, sin, self.q_rot,
                         layer["k_cache"], layer["v_cache"], self.position, self.eps, s.q_heads, s.kv_heads, hd)
            decode_attention(self.q_rot, layer["k_cache"], layer["v_cache"], self.keys, s.q_heads, s.kv_heads, hd,
                             self.attn, self.attn_ws, window=layer["window"])
            layer["prog_o"].run(dependent=True)
            rmsnorm(self.h, layer["o"], self.w_pre_ff[index], self.eps, self.xn, delta_weight=self.w_post_attn[index])
            layer["prog_mlp"].run(dependent=True)
            if index < last:
                rmsnorm(self.h, layer["down"], self.w_in[index + 1], self.eps, self.xn,
                        delta_weight=self.w_post_ff[index])
            else:
                rmsnorm(self.h, layer["down"], self.w_final, self.eps, self.out, delta_weight=self.w_post_ff[index])
        return self.out

    def capture(self) -> None:
        """Record one step (from the current ids) into a CUDA graph; :meth:`replay` then reruns it."""

        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self.step()
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self.step()
        self.graph = graph

    def replay(self) -> torch.Tensor:
        if self.graph is None:
            raise RuntimeError("capture() first")
        self.graph.replay()
        return self.out

    def algorithmic_bytes(self) -> int:
        """Bytes one step must move: packed weights and scales, the KV rows attention reads, norms, embedding rows."""

        s = self.shape
        packed = 0
        for layer in self.layers:
            for prepared in layer["prepared"].values():
                spec = prepared.spec
                packed += (spec.out_features * ((spec.rank + 31) // 32) + spec.rank * ((spec.in_features + 31) // 32)) * 4
                packed += (spec.in_features + spec.rank + spec.out_features) * 2
        kv = 0
        for layer in self.layers:
            rows = 0
            for t in range(self.tokens):
                visible = self.keys + t
                rows = max(rows, min(visible, layer["window"]) if layer["window"] else visible)
            kv += 2 * s.kv_heads * rows * s.head_dim * 2
        norms = len(self.layers) * (4 * s.hidden + 2 * s.head_dim) * 2 + s.hidden * 2
        return packed + kv + norms + self.tokens * s.hidden * 2


def build_gemma3_step(shape: DecoderShape, device: torch.device, *, vocab: int = 262144, tokens: int = 1,
                      position: int = 0, layers: int | None = None, seed: int = 0) -> Gemma3DecodeStep:
    """Random-init packed layers and Gemma shell weights of ``shape`` wired into one decode step."""

    blocks = make_decoder_layers(shape, device, layers=layers, seed=seed)
    shell = random_gemma_shell_weights(shape, vocab, device, layers=len(blocks), seed=seed + 1)
    return Gemma3DecodeStep(shape, blocks, shell, device, tokens=tokens, position=position)


def build_qwen3_step(shape: DecoderShape, device: torch.device, *, vocab: int, tokens: int = 1, position: int = 0,
                     layers: int | None = None, seed: int = 0, sequences: bool = False) -> Qwen3DecodeStep:
    """Random-init packed layers and shell weights of ``shape`` wired into one decode step."""

    blocks = make_decoder_layers(shape, device, layers=layers, seed=seed)
    shell = random_shell_weights(shape, vocab, device, layers=len(blocks), seed=seed + 1)
    return Qwen3DecodeStep(shape, blocks, shell, device, tokens=tokens, position=position, sequences=sequences)


__all__ = [
    "Gemma3DecodeStep",
    "GemmaShellWeights",
    "Qwen3DecodeStep",
    "build_gemma3_step",
    "embedding_bf16",
    "random_gemma_shell_weights",
    "ShellWeights",
    "attention_workspace_bytes",
    "build_qwen3_step",
    "decode_attention",
    "gemv_bf16",
    "qk_norm_rope",
    "random_shell_weights",
    "residual_stats",
    "rmsnorm",
    "rope_tables",
    "silu_mul",
]
