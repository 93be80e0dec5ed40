"""Synthetic decoder-shaped stacks of packed linears (the benchmark workloads).

A decoder layer's packed linears are the q/k/v/o attention projections and the
gate/up/down MLP projections.  :func:`make_decoder_layers` builds random
layout-v1 layers of a given model shape (uniform random sign bits, the scales
``|N(0,1)| * 0.05 + 0.01`` in fp16 for pre and post, ``scale_mid = 1``),
directly on the GPU.  :class:`DecodeChain` runs one decode step through every
layer with the grouped QKV and gate/up calls the reference's model shell uses
(``src/nanoquant/runtime/torch_model.py:311-327, 492-505``).  Its engines:
``"program"`` (default for 1..16 tokens) compiles the whole step into one
persistent :class:`~nanoquant_b200.program.DecodeProgram` launch; ``"calls"``
issues one libnqb call per projection group (optionally captured in a CUDA
graph, like the reference's decode loop).

Rank follows the reference's budget formula at a target bits-per-weight:
``r = floor(bpw * m * n / (m + n))``.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from nanoquant_b200.backend import PreparedLayer, QuantizedLinearSpec
from nanoquant_b200.cuda_backend import (
    CudaPackedSm100Backend,
    Sm100ProjectionGroup,
    grouped_sm100_projection,
    prepare_sm100_projection_group,
)
from nanoquant_b200.packed import PACKED_LAYOUT_VERSION, PackedLayerState, packed_word_count
from nanoquant_b200.program import DecodeProgram, ProgramOp


@dataclass(frozen=True)
class DecoderShape:
    name: str
    layers: int
    hidden: int
    intermediate: int
    q_heads: int
    kv_heads: int
    head_dim: int
    bpw: float = 1.0

    def projections(self) -> dict[str, tuple[int, int]]:
        """projection name -> (in_features, out_features)."""

        q = self.q_heads * self.head_dim
        kv = self.kv_heads * self.head_dim
        return {
            "q_proj": (self.hidden, q),
            "k_proj": (self.hidden, kv),
            "v_proj": (self.hidden, kv),
            "o_proj": (q, self.hidden),
            "gate_proj": (self.hidden, self.intermediate),
            "up_proj": (self.hidden, self.intermediate),
            "down_proj": (self.intermediate, self.hidden),
        }

    def rank(self, n: int, m: int) -> int:
        return int(self.bpw * m * n // (m + n))


QWEN3_8B = DecoderShape("qwen3-8b", 36, 4096, 12288, 32, 8, 128, 1.0)
GEMMA3_1B = DecoderShape("gemma-3-1b", 26, 1152, 6912, 4, 1, 256, 1.0)
LLAMA3_8B_055 = DecoderShape("llama-3-8b", 32, 4096, 14336, 32, 8, 128, 0.55)


def layer_bytes(n: int, m: int, r: int, *, scale_bytes: int = 2) -> int:
    """Algorithmic weight bytes of one packed layer: sign words plus the three scale vectors."""

    return 4 * (m * packed_word_count(r) + r * packed_word_count(n)) + scale_bytes * (n + r + m)


def random_packed_layer(name: str, n: int, m: int, r: int, generator: torch.Generator,
                        device: torch.device) -> PackedLayerState:
    """Uniform random signs as layout-v1 words (tail bits cleared) with config-0 style scales."""

    def words(rows: int, columns: int) -> torch.Tensor:
        per_row = packed_word_count(columns)
        raw = torch.randint(-(2**31), 2**31 - 1, (rows, per_row), generator=generator, dtype=torch.int64,
                            device=device)
        tail = columns % 32
        if tail:
            raw[:, -1] &= (1 << tail) - 1
        return raw.to(torch.int32).contiguous()

    def scales(size: int) -> torch.Tensor:
        return (torch.randn(size, generator=generator, device=device).abs() * 0.05 + 0.01).half()

    spec = QuantizedLinearSpec(name, "nanoquant-v1", n, m, r, "float32", "float16")
    return PackedLayerState(spec, PACKED_LAYOUT_VERSION, words(m, r), words(r, n), scales(n),
                            torch.ones(r, device=device).half(), scales(m))


def random_codebook_layer(name: str, n: int, m: int, r: int, rng: np.random.Generator, *,
                          overlay_fraction: float = 0.01):
    """A product-codebook layer with int8 outlier rows, on the host.

    Every 16-sign group of V is an 8-bit index into one per-layer table of 256
    random 16-bit sign words: a 32-bit word of V is the record ``lo | hi << 8``
    of ``product-codebook-free-k16-v1`` with both half tables equal to that
    table.  The format keeps at least one free row, so row 0 stores its
    table-decoded words plainly (bit-identical).  U is plain packed signs.
    ``ceil(overlay_fraction * m)`` uniformly chosen output rows carry an int8
    residual row (uniform in [-127, 127]) with fp16 row scale 0.002.  Scales
    ``|N(0,1)| * 0.05 + 0.01`` in fp16, ``scale_mid = 1``.
    """

    from nanoquant_b200.overlay import OutlierRowOverlay, OverlaidLayerState
    from nanoquant_b200.product_codebook import (
        PRODUCT_CODEBOOK_FORMAT_VERSION,
        ProductCodebookLayerState,
        pack_product_codebook_indices,
    )

    words_u = packed_word_count(r)
    words_v = packed_word_count(n)
    left = rng.integers(0, 2**32, size=(m, words_u), dtype=np.uint64).astype(np.uint32)
    if r % 32:
        left[:, -1] &= np.uint32((1 << (r % 32)) - 1)
    table = rng.integers(0, 2**16, size=256, dtype=np.uint32).astype(np.uint16)
    records = rng.integers(0, 256, size=(r, words_v, 2), dtype=np.uint32)
    if n % 32:  # signs past the last column are zero: the tail word's groups index an all-zero entry
        raise ValueError("config-4 layers have widths that are multiples of 32")
    record = records[..., 0] | (records[..., 1] << 8)
    free = (table[records[:1, :, 0]].astype(np.uint32) | (table[records[:1, :, 1]].astype(np.uint32) << 16))
    scales = lambda k: torch.from_numpy((np.abs(rng.standard_normal(k)) * 0.05 + 0.01).astype(np.float16))  # noqa
    spec = QuantizedLinearSpec(name, "nanoquant-v1", n, m, r, "float32", "float16")
    half = torch.from_numpy(table.view(np.int16).copy())
    state = ProductCodebookLayerState(
        spec, PRODUCT_CODEBOOK_FORMAT_VERSION, False, 1,
        torch.from_numpy(left.view(np.int32).copy()), torch.from_numpy(free.view(np.int32).copy()),
        pack_product_codebook_indices(torch.from_numpy(record[1:].astype(np.int32))), half, half.clone(),
        scales(n), torch.ones(r, dtype=torch.float16), scales(m))
    rows = max(1, -(-int(round(overlay_fraction * m * 1000)) // 1000))
    ids = np.sort(rng.choice(m, size=rows, replace=False)).astype(np.int32)
    overlay = OutlierRowOverlay(torch.from_numpy(ids), torch.from_numpy(rng.integers(-127, 128, size=(rows, n),
                                                                                     dtype=np.int8)),
                                torch.full((rows,), 0.002, dtype=torch.float16))
    return OverlaidLayerState(state, overlay)


def make_codebook_layers(shape: DecoderShape, *, layers: int | None = None, seed: int = 0) -> list[dict]:
    """Config-4 layers (product-codebook V, int8 outlier rows) of ``shape``, on the host."""

    rng = np.random.default_rng(seed)
    result = []
    for index in range(shape.layers if layers is None else layers):
        result.append({proj: random_codebook_layer(f"blocks.{index}.{proj}", n, m, shape.rank(n, m), rng)
                       for proj, (n, m) in shape.projections().items()})
    return result


def codebook_layer_bytes(n: int, m: int, r: int, overlay_rows: int) -> int:
    """Algorithmic bytes of one config-4 layer: U words, V's 8-bit group indices, the 512-byte table pair, fp16
    scales and the int8 overlay rows with their fp16 scales and int32 ids."""

    return (4 * m * packed_word_count(r) + r * ((n + 15) // 16) + 512 + 2 * (n + r + m)
            + overlay_rows * (n + 6))


def make_decoder_layers(shape: DecoderShape, device: torch.device, *, layers: int | None = None,
                        seed: int = 0) -> list[dict[str, PackedLayerState]]:
    generator = torch.Generator(device=device).manual_seed(seed)
    result = []
    for index in range(shape.layers if layers is None else layers):
        block = {}
        for proj, (n, m) in shape.projections().items():
            block[proj] = random_packed_layer(f"blocks.{index}.{proj}", n, m, shape.rank(n, m), generator, device)
        result.append(block)
    return result


@dataclass
class _PreparedBlock:
    qkv: Sm100ProjectionGroup
    o_proj: PreparedLayer
    gate_up: Sm100ProjectionGroup
    down_proj: PreparedLayer


class DecodeChain:
    """All packed linears of a decoder, run for one decode step (batch ``tokens``)."""

    def __init__(self, shape: DecoderShape, blocks: list[dict[str, PackedLayerState]], device: torch.device,
                 tokens: int = 1, engine: str | None = None,
                 backend: CudaPackedSm100Backend | None = None) -> None:
        if engine is None:
            engine = "program" if tokens <= 16 else "calls"
        if engine not in ("program", "calls"):
            raise ValueError(f"unknown engine {engine!r}")
        if engine == "program" and tokens > 16:
            raise ValueError("the program engine takes 1..16 tokens")
        self.shape = shape
        self.device = device
        self.tokens = tokens
        self.engine = engine
        self.backend = backend if backend is not None else CudaPackedSm100Backend()
        self.blocks: list[_PreparedBlock] = []
        first = blocks[0] if blocks else {}
        self.codebook_rows = ({proj: int(state.overlay.row_ids.numel()) for proj, state in first.items()}
                              if first and all(hasattr(state, "overlay") for state in first.values()) else None)
        for block in blocks:
            prepared = {name: self.backend.prepare(state, device) for name, state in block.items()}
            qkv = prepare_sm100_projection_group((prepared["q_proj"], prepared["k_proj"], prepared["v_proj"]))
            gate_up = prepare_sm100_projection_group((prepared["gate_proj"], prepared["up_proj"]))
            if qkv is None or gate_up is None:
                raise RuntimeError("grouped projections could not be prepared")
            self.blocks.append(_PreparedBlock(qkv, prepared["o_proj"], gate_up, prepared["down_proj"]))
        projections = shape.projections()
        hidden_in = torch.randn(tokens, shape.hidden, device=device).bfloat16()
        self.inputs = {
            "hidden": hidden_in,
            "attn": torch.randn(tokens, projections["o_proj"][0], device=device).bfloat16(),
            "mlp": torch.randn(tokens, shape.hidden, device=device).bfloat16(),
            "act": torch.randn(tokens, shape.intermediate, device=device).bfloat16(),
        }
        self.graph: torch.cuda.CUDAGraph | None = None
        self.graph_output: torch.Tensor | None = None
        self.program: DecodeProgram | None = None
        if engine == "program":
            ops = []
            for block in self.blocks:
                ops += [ProgramOp(block.qkv.layers, self.inputs["hidden"]),
                        ProgramOp((block.o_proj,), self.inputs["attn"]),
                        ProgramOp(block.gate_up.layers, self.inputs["mlp"]),
                        ProgramOp((block.down_proj,), self.inputs["act"])]
            self.program = DecodeProgram(ops)

    @property
    def launches_per_step(self) -> int:
        """libnqb kernel launches of one step.

        Program engine: one launch per step.  Per-call decode (tensor-core
        path): two stage kernels per call, four calls per layer.  Prefill: per
        call and stage one activation pre-pass and one GEMM kernel.
        """

        if self.program is not None:
            return 1
        if self.tokens <= 16:
            return 8 * len(self.blocks)
        return 16 * len(self.blocks)

    def algorithmic_flops(self) -> int:
        """Multiply-adds x 2 of the two sign GEMMs of every linear: 2*r*(m+n) per token."""

        total = 0
        for n, m in self.shape.projections().values():
            total += 2 * self.shape.rank(n, m) * (m + n) * self.tokens
        return total * len(self.blocks)

    def algorithmic_bytes(self) -> int:
        """Weight bytes plus activation traffic (bf16 in, fp32 out) of one step.

        Config-4 layers (product-codebook V with outlier rows) count their
        compact format: U words, V's group indices, tables, scales and rows.
        """

        total = 0
        for proj, (n, m) in self.shape.projections().items():
            r = self.shape.rank(n, m)
            if self.codebook_rows is not None:
                total += codebook_layer_bytes(n, m, r, self.codebook_rows[proj]) + self.tokens * (2 * n + 4 * m)
            else:
                total += layer_bytes(n, m, r) + self.tokens * (2 * n + 4 * m)
        return total * len(self.blocks)

    def step(self) -> torch.Tensor:
        if self.program is not None:
            return self.program.run()[-1][0]
        out = None
        for block in self.blocks:
            grouped_sm100_projection(self.inputs["hidden"], block.qkv)
            self.backend.linear(self.inputs["attn"], block.o_proj)
            grouped_sm100_projection(self.inputs["mlp"], block.gate_up)
            out = self.backend.linear(self.inputs["act"], block.down_proj)
        assert out is not None
        return out

    def capture(self) -> None:
        """Record :meth:`step` into a CUDA graph (after one eager warm-up on a side stream)."""

        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self.step()
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self.graph_output = self.step()
        self.graph = graph

    def replay(self) -> torch.Tensor:
        if self.graph is None or self.graph_output is None:
            raise RuntimeError("capture() first")
        self.graph.replay()
        return self.graph_output
