"""Benchmark of NanoQuant's packed binary low-rank linear on B200: one JSON line.

Default workload ``decode`` (the metric's own config): one
decode token (batch 1) through the full Qwen3-8B-shaped decoder step -- 36
layers of RMSNorm, packed q/k/v/o/gate/up/down projections at ~1 bpw (layout
v1 words, fp16 scales), q/k norm + RoPE, grouped-query attention over 2048
cached bf16 tokens, SwiGLU, the final norm and the 151936 x 4096 bf16 lm
head -- replayed from one CUDA graph.  Weights are random (2.4 GB per step,
larger than the 126 MB L2, so no L2 flush is needed); inputs are synthetic.

The same line carries:
* ``roofline`` for the dominant kernel, the persistent decode program that
  runs the packed linears: the step's 252 packed linears as one program
  launch, timed with CUDA events (algorithmic bytes per launch / launch time);
  ``step_roofline`` is the whole step's bytes over the step time;
* ``e2e``: the same step through the public API with the token's hidden
  state copied in from pinned host memory and the logits copied back;
* ``cpu_baseline``: the reference's CPU path for the same step (the oracle
  port of ``PackedReferenceBackend`` and the model shell) on the host cores;
* ``prefill``: BASELINE config 3 (Llama-3-8B, 0.55 bpw, 8 x 4096 tokens) by
  disjoint token batches over the ranks, and with ``N > 1`` ``row_shard``:
  one 4096-token sequence with every linear's U rows split over the ranks and
  the output slices all-gathered over NCCL.

Other workloads (``--workload``): ``decode-bs16`` (config 2 at batch 16: 16
independent sequences, each on its own cache), ``decode-16tok`` (16 new
tokens of one sequence),
``gemma1b`` (config 1: the full Gemma-3-1B-shaped step from token ids),
``linears`` / ``linears-bs16`` (the packed linears alone), ``prefill``
(config 3 alone), ``single-linear`` (config 0, ``--tokens`` 1 or 8) and
``single-linear-stacked`` (config 0 x 1024 layers in one program).

Launch: ``python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--workload W]``;
for N > 1 under ``torch.distributed.run``: decode does not shard, so every
rank runs an independent replica ("replicas only") and ``value`` sums them;
the prefill token batches split the 8 x 4096 tokens over the ranks.
``--impl reference`` times the CPU path alone (rank 0; other ranks exit).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tok/s (bs1, Qwen3-8B shape ~1 bpw); packed-GEMV HBM GB/s vs peak"
UNIT = "tok/s"
STEP_VOCAB, STEP_POSITION = 151936, 2048
GEMMA_POSITION = 1024
STACKED_LAYERS = 1024  # config-0 layers in the stacked workload's program
PREFILL_TOKENS = 8 * 4096


def _peak_table() -> dict[str, tuple[float, str]]:
    """HBM GB/s and sustained dense bf16 TFLOP/s: measured on this pool, else the fallback figures."""

    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm": (float(data["hbm_gbs"]), "measured"),
                "tensor": (float(data.get("bf16_tflops_sustained", data["bf16_tflops"])), "measured-sustained")}
    return {"hbm": (6650.0, "fallback"), "tensor": (1400.0, "fallback-sustained")}


def _cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int) -> None:
        self.index = index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def __enter__(self) -> "ClockSampler":
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc) -> None:
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        self.file.flush()
        rows = []
        try:
            for line in Path(self.file.name).read_text().splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        finally:
            os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        sm_max = max(float(r[2]) for r in rows if r[2].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": sm_max, "reasons": reasons,
                "samples": len(rows)}


def _device_status() -> int:
    """libnqb's device status word (NQB_OK = 0; NQB_ERR_TIMEOUT when a bounded wait gave up)."""

    import ctypes

    from nanoquant_b200 import _native

    value = ctypes.c_int32(-1)
    _native.call("nqb_device_status", ctypes.byref(value))
    return value.value


# ----------------------------------------------------------- CPU baseline ---

def _qwen3_cpu_step(tokens: int, layers: int = 36, sequences: bool = False):
    from nanoquant_b200.decode_chain import QWEN3_8B as s
    from oracle.decoder_oracle import CpuDecodeStep

    return CpuDecodeStep(layers=layers, hidden=s.hidden, intermediate=s.intermediate, q_heads=s.q_heads,
                         kv_heads=s.kv_heads, head_dim=s.head_dim, vocab=STEP_VOCAB, position=STEP_POSITION,
                         tokens=tokens, pool=1, sequences=sequences)


def cpu_step_baseline(tokens: int, steps: int = 1, warmup: int = 1, budget_s: float = 240.0,
                      sequences: bool = False) -> dict:
    """The reference's CPU path for the full step: ``warmup`` untimed then ``steps`` timed full steps.

    Every step runs all 36 layers and the lm head.  When ``warmup + steps``
    full steps would exceed ``budget_s``, each step runs only a prefix of the
    layers (the sample string says how many) and its time is scaled to 36.
    """

    setup = time.perf_counter()
    cpu = _qwen3_cpu_step(tokens, sequences=sequences)
    setup_s = time.perf_counter() - setup
    start = time.perf_counter()
    cpu.step()  # first warm-up step, also the estimate
    first = time.perf_counter() - start
    full_layers = cpu.layers
    if first * (warmup + steps) > budget_s:
        cpu.layers = max(1, int(full_layers * budget_s / (first * (warmup + steps))))
    for _ in range(max(0, warmup - 1)):
        cpu.step()
    start = time.perf_counter()
    for _ in range(steps):
        cpu.step()
    per_step = (time.perf_counter() - start) / steps
    head_note = ""
    if cpu.layers != full_layers:
        # scale the layer part to all layers; the lm head runs once per step either way
        per_step = per_step * full_layers / cpu.layers
        head_note = f" (each step ran {cpu.layers} of {full_layers} layers + the lm head; time scaled to all layers)"
    threads = _cpu_threads()
    return {
        "value": tokens / per_step, "unit": UNIT, "cores": threads, "kind": "port",
        "cpu_model": _cpu_model(), "ms_per_step": per_step * 1e3, "steps": steps, "warmup": warmup,
        "sample": f"full qwen3-8b decode step, {tokens} token(s)"
                  f"{' of independent sequences' if sequences else ''}: 36 layers of the oracle port of "
                  f"PackedReferenceBackend.linear (fp32 numpy/BLAS on dense +/-1 signs unpacked once) and the model "
                  f"shell (norms, q/k norm + rope, attention over {STEP_POSITION + 1} cached rows, swiglu), final "
                  f"norm and the {STEP_VOCAB} x 4096 lm head; {threads} host threads ({_cpu_model()}); {steps} timed "
                  f"step(s) after {warmup} warm-up{head_note}; setup {setup_s:.0f} s untimed",
    }


def cpu_gemma_baseline(tokens: int, steps: int = 3, warmup: int = 1) -> dict:
    """The reference's CPU path for the full Gemma-3-1B step (26 layers, no vocabulary head)."""

    from nanoquant_b200.decode_chain import GEMMA3_1B as s
    from oracle.decoder_oracle import CpuDecodeStep

    cpu = CpuDecodeStep(layers=s.layers, hidden=s.hidden, intermediate=s.intermediate, q_heads=s.q_heads,
                        kv_heads=s.kv_heads, head_dim=s.head_dim, vocab=0, position=GEMMA_POSITION, tokens=tokens,
                        pool=2, family="gemma")
    for _ in range(warmup):
        cpu.step()
    start = time.perf_counter()
    for _ in range(steps):
        cpu.step()
    per_step = (time.perf_counter() - start) / steps
    threads = _cpu_threads()
    return {"value": tokens / per_step, "unit": UNIT, "cores": threads, "kind": "port", "cpu_model": _cpu_model(),
            "ms_per_step": per_step * 1e3, "steps": steps, "warmup": warmup,
            "sample": f"full gemma-3-1b decode step, {tokens} token(s): 26 layers of the oracle port of "
                      f"PackedReferenceBackend.linear (fp32, two distinct layers' weights cycled) and the Gemma-3 "
                      f"shell (sandwich norms, q/k norm + rope, windowed attention over {GEMMA_POSITION + 1} rows, "
                      f"gated gelu), final norm; {threads} host threads ({_cpu_model()}); {steps} timed steps"}


def cpu_codebook_baseline(tokens: int, sample_layers: int = 2, repeats: int = 3) -> dict:
    """The oracle (product-codebook decode to layout v1 at prepare, then the reference's packed linear plus the
    int8 row overlay) on ``sample_layers`` config-4 layers, scaled to 26 layers."""

    import numpy as np

    from nanoquant_b200.decode_chain import GEMMA3_1B, make_codebook_layers
    from oracle import packed_oracle as po

    blocks = make_codebook_layers(GEMMA3_1B, layers=sample_layers, seed=0)
    rng = np.random.default_rng(1)
    layers = []
    for block in blocks:
        for state in block.values():
            packed = state.base.to_packed()
            layer = po.OracleLayer(
                packed.spec.in_features, packed.spec.out_features, packed.spec.rank, packed.left_words.numpy(),
                packed.right_words.numpy(), packed.scale_pre.float().numpy(), packed.scale_mid.float().numpy(),
                packed.scale_post.float().numpy())
            layer.overlay_row_ids = state.overlay.row_ids.numpy()
            layer.overlay_values = state.overlay.values.numpy()
            layer.overlay_scales = state.overlay.scales.float().numpy()
            layer.prepared()
            layers.append((layer, rng.standard_normal((tokens, layer.in_features)).astype(np.float32)))
    for layer, x in layers:
        po.packed_linear(x, layer)
    start = time.perf_counter()
    for _ in range(repeats):
        for layer, x in layers:
            po.packed_linear(x, layer)
    step = (time.perf_counter() - start) / repeats * GEMMA3_1B.layers / sample_layers
    threads = _cpu_threads()
    return {"value": tokens / step, "unit": UNIT, "cores": threads, "kind": "port", "ms_per_step": step * 1e3,
            "cpu_model": _cpu_model(),
            "sample": f"{sample_layers} of 26 config-4 layers x 7 projections, {tokens} token(s), {repeats} reps: the "
                      f"oracle port (codebook decoded at prepare, fp32 packed linear, int8 row overlay) on {threads} "
                      f"host threads ({_cpu_model()}); scaled to 26 layers"}


def cpu_linear_baseline(n: int, m: int, r: int, tokens: int, repeats: int = 200, layers: int = 1) -> dict:
    """The oracle port of ``PackedReferenceBackend.linear`` on one config-0 layer.

    ``layers`` > 1 states the rate for a step through that many such layers
    (the stacked workload): the per-call time of one layer times ``layers``.
    """

    import numpy as np

    from oracle import packed_oracle as po

    rng = np.random.default_rng(0)

    def words(rows, cols):
        raw = rng.integers(0, 2**32, size=(rows, po.word_count(cols)), dtype=np.uint64).astype(np.uint32)
        if cols % 32:
            raw[:, -1] &= np.uint32((1 << (cols % 32)) - 1)
        return raw.view(np.int32)

    scale = lambda k: (np.abs(rng.standard_normal(k)) * 0.05 + 0.01).astype(np.float16).astype(np.float32)  # noqa: E731
    layer = po.OracleLayer(n, m, r, words(m, r), words(r, n), scale(n), np.ones(r, np.float32), scale(m))
    layer.prepared()
    x = rng.standard_normal((tokens, n)).astype(np.float32)
    for _ in range(3):
        po.packed_linear(x, layer)
    start = time.perf_counter()
    for _ in range(repeats):
        po.packed_linear(x, layer)
    per = (time.perf_counter() - start) / repeats
    threads = _cpu_threads()
    scaled = f"; scaled to a step through {layers} layers" if layers > 1 else ""
    return {"value": tokens / (per * layers), "unit": UNIT, "cores": threads, "kind": "port",
            "ms_per_step": per * layers * 1e3, "cpu_model": _cpu_model(),
            "sample": f"one {n}->{m} r{r} layer, {tokens} token(s), {repeats} calls of the oracle port of "
                      f"PackedReferenceBackend.linear (fp32) on {threads} host threads ({_cpu_model()}){scaled}"}


def cpu_prefill_baseline(tokens: int = 128) -> dict:
    """The oracle port on 1 of 32 Llama-3-8B (0.55 bpw) layers at ``tokens`` tokens, scaled to 32 layers."""

    import numpy as np

    from nanoquant_b200.decode_chain import LLAMA3_8B_055 as shape
    from oracle import packed_oracle as po

    rng = np.random.default_rng(0)
    layers = {}
    for proj, (n, m) in shape.projections().items():
        r = shape.rank(n, m)
        left = rng.integers(0, 2**32, size=(m, po.word_count(r)), dtype=np.uint64).astype(np.uint32)
        right = rng.integers(0, 2**32, size=(r, po.word_count(n)), dtype=np.uint64).astype(np.uint32)
        if r % 32:
            left[:, -1] &= np.uint32((1 << (r % 32)) - 1)
        if n % 32:
            right[:, -1] &= np.uint32((1 << (n % 32)) - 1)
        layer = po.OracleLayer(n, m, r, left.view(np.int32), right.view(np.int32),
                               np.full(n, 0.03, np.float32), np.ones(r, np.float32), np.full(m, 0.03, np.float32))
        layer.prepared()
        layers[proj] = layer
    xs = {proj: rng.standard_normal((tokens, n)).astype(np.float32) for proj, (n, _m) in shape.projections().items()}
    start = time.perf_counter()
    for proj, layer in layers.items():
        po.packed_linear(xs[proj], layer)
    per_layer = time.perf_counter() - start
    step = per_layer * shape.layers
    threads = _cpu_threads()
    return {"value": tokens / step, "unit": UNIT, "cores": threads, "kind": "port", "ms_per_step": step * 1e3,
            "cpu_model": _cpu_model(),
            "sample": f"1 of 32 llama-3-8b layers (7 projections, 0.55 bpw), {tokens} tokens, oracle port of "
                      f"PackedReferenceBackend.linear (fp32) on {threads} host threads ({_cpu_model()}); "
                      f"scaled to 32 layers"}


# --------------------------------------------------------------- runners ---

class StepRunner:
    """The full Qwen3-8B-shaped decode step (``nanoquant_b200.decoder``), replayed from a CUDA graph."""

    bound = "hbm"

    def __init__(self, device, tokens: int, layers: int | None, sequences: bool = False) -> None:
        from nanoquant_b200.decode_chain import QWEN3_8B
        from nanoquant_b200.decoder import build_qwen3_step

        self.step_obj = build_qwen3_step(QWEN3_8B, device, vocab=STEP_VOCAB, tokens=tokens, position=STEP_POSITION,
                                         layers=layers, sequences=sequences)
        self.tokens = tokens
        self.layers = len(self.step_obj.layers)
        self.input = self.step_obj.hidden_in
        self.launches_per_step = self.step_obj.kernel_launches()
        self.step_obj.capture()

    def run(self):
        return self.step_obj.replay()

    def algorithmic_bytes(self) -> int:
        return self.step_obj.algorithmic_bytes()


class GemmaStepRunner:
    """The full Gemma-3-1B-shaped decode step (config 1) from token ids, replayed from a CUDA graph."""

    bound = "hbm"

    def __init__(self, device, tokens: int, layers: int | None) -> None:
        import torch

        from nanoquant_b200.decode_chain import GEMMA3_1B
        from nanoquant_b200.decoder import build_gemma3_step

        self.step_obj = build_gemma3_step(GEMMA3_1B, device, tokens=tokens, position=GEMMA_POSITION, layers=layers)
        self.tokens = tokens
        self.layers = len(self.step_obj.layers)
        self.input = self.step_obj.ids
        self.step_obj.ids.copy_(torch.arange(tokens, device=device) * 97 + 11)
        self.launches_per_step = self.step_obj.kernel_launches()
        self.step_obj.capture()

    def host_input(self):
        import torch

        return (torch.arange(self.tokens) * 131 + 5).to(torch.int64)

    def run(self):
        return self.step_obj.replay()

    def algorithmic_bytes(self) -> int:
        return self.step_obj.algorithmic_bytes()


class ChainRunner:
    """Packed linears only (``DecodeChain``): one persistent program launch per step, or per-call kernels."""

    bound = "hbm"

    def __init__(self, shape, device, tokens: int, layers: int | None, engine: str | None = None) -> None:
        from nanoquant_b200.decode_chain import DecodeChain, make_decoder_layers

        self.chain = DecodeChain(shape, make_decoder_layers(shape, device, layers=layers, seed=0), device,
                                 tokens=tokens, engine=engine)
        self.tokens = tokens
        self.layers = len(self.chain.blocks)
        self.input = self.chain.inputs["hidden"]
        self.launches_per_step = self.chain.launches_per_step
        if self.chain.program is None:
            self.chain.capture()

    def run(self):
        return self.chain.step() if self.chain.program is not None else self.chain.replay()

    def algorithmic_bytes(self) -> int:
        return self.chain.algorithmic_bytes()


class CodebookRunner:
    """BASELINE config 4 on Gemma-3-1B shapes: 26 layers x 7 product-codebook linears with int8 outlier rows.

    ``tokens`` <= 16: one persistent program per step (decode); more: the
    per-call tensor-core prefill kernels.
    """

    def __init__(self, device, tokens: int, layers: int | None) -> None:
        from nanoquant_b200.decode_chain import GEMMA3_1B, DecodeChain, make_codebook_layers

        engine = "program" if tokens <= 16 else "calls"
        self.bound = "hbm" if tokens <= 16 else "tensor"
        self.chain = DecodeChain(GEMMA3_1B, make_codebook_layers(GEMMA3_1B, layers=layers, seed=0), device,
                                 tokens=tokens, engine=engine)
        self.tokens = tokens
        self.layers = len(self.chain.blocks)
        self.input = self.chain.inputs["hidden"]
        self.launches_per_step = self.chain.launches_per_step

    def run(self):
        return self.chain.step()

    def algorithmic_bytes(self) -> int:
        return self.chain.algorithmic_bytes()

    def algorithmic_flops(self) -> int:
        return self.chain.algorithmic_flops()


class PrefillRunner:
    """Llama-3-8B (0.55 bpw) packed linears on ``tokens`` tokens per rank (tensor-core prefill kernels)."""

    bound = "tensor"

    def __init__(self, device, tokens: int, layers: int | None) -> None:
        from nanoquant_b200.decode_chain import LLAMA3_8B_055, DecodeChain, make_decoder_layers

        self.chain = DecodeChain(LLAMA3_8B_055, make_decoder_layers(LLAMA3_8B_055, device, layers=layers, seed=0),
                                 device, tokens=tokens, engine="calls")
        self.tokens = tokens
        self.layers = len(self.chain.blocks)
        self.input = self.chain.inputs["hidden"]
        self.launches_per_step = self.chain.launches_per_step

    def run(self):
        return self.chain.step()

    def algorithmic_flops(self) -> int:
        return self.chain.algorithmic_flops()


class SingleLinearRunner:
    """BASELINE config 0 (640 -> 2048, rank 480): one ``CudaPackedSm100Backend.linear`` call, captured in a graph."""

    bound = "hbm"

    def __init__(self, device, tokens: int) -> None:
        import torch

        from nanoquant_b200 import CudaPackedSm100Backend
        from nanoquant_b200.decode_chain import layer_bytes, random_packed_layer

        n, m, r = 640, 2048, 480
        g = torch.Generator(device=device).manual_seed(0)
        self.backend = CudaPackedSm100Backend()
        self.layer = self.backend.prepare(random_packed_layer("blocks.0.mlp.up_proj", n, m, r, g, device), device)
        self.input = torch.randn(tokens, n, generator=g, device=device).bfloat16()
        self.tokens, self.layers, self.launches_per_step = tokens, 1, 2
        self._bytes = layer_bytes(n, m, r) + tokens * (2 * n + 4 * m)
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            self.backend.linear(self.input, self.layer)  # warm-up outside capture (workspace, smem attributes)
        torch.cuda.current_stream(device).wait_stream(side)
        torch.cuda.synchronize(device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.output = self.backend.linear(self.input, self.layer)

    def run(self):
        self.graph.replay()
        return self.output

    def algorithmic_bytes(self) -> int:
        return self._bytes


class StackedLinearRunner:
    """BASELINE config 0 (2048 x 640, rank 480) as ``count`` independent layers run as one program."""

    bound = "hbm"

    def __init__(self, device, tokens: int, count: int) -> None:
        import torch

        from nanoquant_b200 import CudaPackedSm100Backend
        from nanoquant_b200.decode_chain import layer_bytes, random_packed_layer
        from nanoquant_b200.program import DecodeProgram, ProgramOp

        n, m, r = 640, 2048, 480
        g = torch.Generator(device=device).manual_seed(0)
        backend = CudaPackedSm100Backend()
        self.input = torch.randn(tokens, n, generator=g, device=device).bfloat16()
        self.layers_prepared = [backend.prepare(random_packed_layer(f"stack.{i}.up_proj", n, m, r, g, device), device)
                                for i in range(count)]
        # the layers share their input: three per program op (one grouped projection)
        group = 3
        self.program = DecodeProgram([ProgramOp(tuple(self.layers_prepared[i:i + group]), self.input)
                                      for i in range(0, count, group)])
        self.tokens = tokens
        self.layers = count
        self.launches_per_step = 1
        self._bytes = count * (layer_bytes(n, m, r) + tokens * (2 * n + 4 * m))

    def run(self):
        return self.program.run()[-1][0]

    def algorithmic_bytes(self) -> int:
        return self._bytes


WORKLOADS = {
    "decode": {"kind": "step", "metric": METRIC, "tokens": 1,
               "description": "qwen3-8b decode step bs1 ({layers} layers: norms, packed q/k/v/o/gate/up/down, q/k "
                              "norm + rope, attention over 2048 cached tokens, swiglu; final norm; bf16 lm head "
                              "151936 x 4096)",
               "model": "qwen3-8b-shape random-init: packed weights ~1 bpw (layout v1, fp16 scales), bf16 norms and "
                        "lm head, bf16 kv cache N(0,1)"},
    "decode-bs16": {"kind": "step", "metric": "decode tok/s (bs16, Qwen3-8B shape ~1 bpw); HBM GB/s vs peak",
                    "tokens": 16, "sequences": True,
                    "description": "qwen3-8b decode step bs16 ({layers} layers, full shell and lm head): 16 "
                                   "independent sequences, each the next token on its own 2048-token cache",
                    "model": "qwen3-8b-shape random-init, as decode"},
    "decode-16tok": {"kind": "step", "metric": "decode tok/s (16 new tokens of one sequence, Qwen3-8B shape ~1 bpw); "
                                               "HBM GB/s vs peak",
                     "tokens": 16,
                     "description": "qwen3-8b decode step of 16 new tokens of one sequence ({layers} layers, full "
                                    "shell and lm head) on its 2048-token cache (KV rows read once per step)",
                     "model": "qwen3-8b-shape random-init, as decode"},
    "gemma1b": {"kind": "gemma", "metric": "decode tok/s (bs1, Gemma-3-1B shape ~1 bpw); HBM GB/s vs peak",
                "tokens": 1,
                "description": "gemma-3-1b decode step bs1 ({layers} layers: bf16 embedding, sandwich norms, packed "
                               "q/k/v/o/gate/up/down, q/k norm + rope, attention over 1024 cached tokens (512-key "
                               "window on local layers), gated gelu; final norm; no vocabulary head)",
                "model": "gemma-3-1b-shape random-init: packed weights ~1 bpw (layout v1, fp16 scales), bf16 norms "
                         "1+N(0,0.02) and embedding, bf16 kv cache N(0,1)"},
    "linears": {"kind": "linears", "metric": "packed-linear decode tok/s (bs1, Qwen3-8B shape ~1 bpw); HBM GB/s",
                "tokens": 1,
                "description": "qwen3-8b packed linears only, decode bs1 ({layers} layers x q,k,v,o,gate,up,down; "
                               "grouped qkv and gate/up)",
                "model": "qwen3-8b-shape random-init packed weights ~1 bpw"},
    "linears-bs16": {"kind": "linears", "metric": "packed-linear decode tok/s (bs16, Qwen3-8B shape); HBM GB/s",
                     "tokens": 16,
                     "description": "qwen3-8b packed linears only, decode bs16 ({layers} layers)",
                     "model": "qwen3-8b-shape random-init packed weights ~1 bpw"},
    "prefill": {"kind": "prefill",
                "metric": "prefill tok/s (Llama-3-8B shape 0.55 bpw, 8x4096 tokens); tensor TFLOP/s vs peak",
                "description": "llama-3-8b packed linears, prefill 8x4096 tokens ({layers} layers x "
                               "q,k,v,o,gate,up,down)",
                "model": "llama-3-8b-shape random-init packed weights 0.55 bpw"},
    "codebook-decode": {"kind": "codebook", "metric": "codebook decode tok/s (bs1, Gemma-3-1B shapes, product-"
                                                      "codebook V + 1% int8 rows); HBM GB/s",
                        "tokens": 1,
                        "description": "gemma-3-1b product-codebook packed linears with int8 outlier rows, decode bs1 "
                                       "({layers} layers x q,k,v,o,gate,up,down in one program; V streamed as "
                                       "16-bit records and decoded in stage 1)",
                        "model": "config 4: 8-bit group indices into one 256-entry 16-bit table per layer, plain U, "
                                 "1% int8 rows (scale 0.002)"},
    "codebook-prefill": {"kind": "codebook", "metric": "codebook prefill tok/s (bs64, Gemma-3-1B shapes, product-"
                                                       "codebook V + 1% int8 rows); TFLOP/s",
                         "tokens": 64,
                         "description": "gemma-3-1b product-codebook packed linears with int8 outlier rows, prefill 64 "
                                        "tokens ({layers} layers x q,k,v,o,gate,up,down, tensor-core kernels)",
                         "model": "config 4 (as codebook-decode)"},
    "single-linear": {"kind": "single", "metric": "single packed linear tok/s (2048x640 r480); HBM GB/s",
                      "tokens": 1,
                      "description": "one 640->2048 rank-480 packed linear (config 0), {tokens} token(s)",
                      "model": "config 0: iid sign words, fp16 scales |N(0,1)|*0.05+0.01, bf16 x N(0,1)"},
    "single-linear-stacked": {"kind": "stacked",
                              "metric": "stacked packed linears tok/s (1024 x 2048x640 r480); HBM GB/s",
                              "tokens": 1,
                              "description": "1024 independent 640->2048 rank-480 layers (config 0) on one input "
                                             "in one program, three per op, {tokens} token(s)",
                              "model": "config 0 x 1024 (165 MB of weights, larger than L2)"},
}


def _build(name: str, device, tokens: int, layers: int | None, engine: str | None):
    from nanoquant_b200 import decode_chain

    kind = WORKLOADS[name]["kind"]
    if kind == "step":
        return StepRunner(device, tokens, layers, WORKLOADS[name].get("sequences", False))
    if kind == "gemma":
        return GemmaStepRunner(device, tokens, layers)
    if kind == "codebook":
        return CodebookRunner(device, tokens, layers)
    if kind == "linears":
        return ChainRunner(decode_chain.QWEN3_8B, device, tokens, layers, engine)
    if kind == "prefill":
        return PrefillRunner(device, tokens, layers)
    if kind == "single":
        return SingleLinearRunner(device, tokens)
    return StackedLinearRunner(device, tokens, STACKED_LAYERS)


# ----------------------------------------------------------------- timing ---

class Timer:
    """Times ``steps`` runs of a callable on the device: barrier + synchronize on both sides, max over ranks."""

    def __init__(self, device, world: int) -> None:
        self.device, self.world = device, world

    def barrier(self) -> None:
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier()

    def max_over_ranks(self, *values: float) -> list[float]:
        if self.world == 1:
            return list(values)
        import torch
        import torch.distributed as dist

        t = torch.tensor(values, dtype=torch.float64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return [float(v) for v in t.tolist()]

    def time(self, run, steps: int, warmup: int, clocks_index: int | None = None) -> tuple[float, dict | None]:
        import torch

        for _ in range(warmup):
            run()
        torch.cuda.synchronize(self.device)
        stream = torch.cuda.current_stream(self.device)
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        sampler = ClockSampler(clocks_index) if clocks_index is not None else None
        if sampler is not None:
            sampler.__enter__()
        try:
            self.barrier()
            torch.cuda.synchronize(self.device)
            start.record(stream)
            for _ in range(steps):
                run()
            stop.record(stream)
            torch.cuda.synchronize(self.device)
            self.barrier()
        finally:
            if sampler is not None:
                sampler.__exit__()
        (elapsed,) = self.max_over_ranks(start.elapsed_time(stop))
        return elapsed / steps, (sampler.summary() if sampler is not None else None)


def _time_step_program(step, steps: int, warmup: int, timer: Timer) -> dict:
    """Mean device time of the step's program launch: CUDA events around each launch (the residual copy and
    statistics kernels before it run outside the event pair), max over ranks."""

    import torch

    from nanoquant_b200.decoder import residual_stats

    stream = torch.cuda.current_stream(step.device)
    pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i in range(warmup + steps):
        step.h.copy_(step.hidden_in)
        residual_stats(step.h, step.stats)
        if i >= warmup:
            pairs[i - warmup][0].record(stream)
        step.program.run()
        if i >= warmup:
            pairs[i - warmup][1].record(stream)
    torch.cuda.synchronize(step.device)
    _check_status("the step-program timing")
    (ms,) = timer.max_over_ranks(sum(a.elapsed_time(b) for a, b in pairs) / steps)
    return {"ms": ms, "bytes": step.program_bytes(), "launches": steps}


def _check_status(where: str) -> None:
    status = _device_status()
    if status != 0:
        raise SystemExit(f"libnqb device status {status} after {where} (a bounded wait gave up)")


def _hbm_roofline(bytes_per: int, ms: float, peaks: dict, scope: str) -> dict:
    achieved = bytes_per / (ms * 1e-3) / 1e9
    return {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm"][0], "unit": "GB/s",
            "frac": achieved / peaks["hbm"][0], "traffic": None, "peak_kind": peaks["hbm"][1],
            "algorithmic_bytes_per_launch": bytes_per, "launch_ms": ms, "scope": scope}


def _tensor_roofline(flops: int, ms: float, peaks: dict, scope: str) -> dict:
    achieved = flops / (ms * 1e-3) / 1e12
    return {"bound": "tensor", "achieved": achieved, "peak": peaks["tensor"][0], "unit": "TFLOP/s",
            "frac": achieved / peaks["tensor"][0], "traffic": None, "peak_kind": peaks["tensor"][1],
            "algorithmic_flops_per_step_per_gpu": flops, "scope": scope}


def _prefill_extra(device, timer: Timer, world: int, rank: int, peaks: dict) -> dict:
    """Config 3 by disjoint token batches: rank g takes 32768 / N tokens of the 8 x 4096 (no collective)."""

    import torch

    from nanoquant_b200.sharding import token_range

    lo, hi = token_range(PREFILL_TOKENS, world, rank)
    runner = PrefillRunner(device, hi - lo, None)
    ms, _ = timer.time(runner.run, 3, 3)
    _check_status("the prefill token batches")
    flops = runner.algorithmic_flops()
    del runner
    torch.cuda.empty_cache()
    return {"value": PREFILL_TOKENS * 1000.0 / ms, "unit": UNIT, "ms_per_step": ms, "n_gpus": world,
            "parallelism": f"token-batches{world}", "tokens_per_gpu": hi - lo, "scaling": "strong",
            "config": "llama-3-8b 0.55 bpw, 32 layers x 7 packed linears, 8 x 4096 tokens split over the ranks",
            "roofline": _tensor_roofline(flops, ms, peaks, "per-GPU packed-linear flops / step time")}


def _row_shard_extra(device, timer: Timer, world: int, rank: int) -> dict:
    """One 4096-token sequence through 32 Llama-3-8B layers with every linear's U rows split over the ranks.

    Each linear runs stage 1 in full and stage 2 on this rank's rows, then
    all-gathers the fp32 output slices (NCCL, on a side stream); the next
    linear's kernels overlap that gather.
    """

    import torch

    from nanoquant_b200 import CudaPackedSm100Backend
    from nanoquant_b200.decode_chain import LLAMA3_8B_055 as shape
    from nanoquant_b200.decode_chain import make_decoder_layers
    from nanoquant_b200.sharding import RowShardedLinear

    tokens = 4096
    backend = CudaPackedSm100Backend()
    blocks = make_decoder_layers(shape, device, seed=0)
    side = torch.cuda.Stream(device)  # one gather stream: NCCL serialises a communicator's collectives anyway
    linears = [RowShardedLinear(backend, state, device, stream=side) for block in blocks for state in block.values()]
    del blocks
    g = torch.Generator(device=device).manual_seed(3)
    inputs = {n: torch.randn(tokens, n, generator=g, device=device).bfloat16()
              for n in {lin.local.spec.in_features for lin in linears}}

    def run():
        works = [lin.start(inputs[lin.local.spec.in_features]) for lin in linears]
        for work in works:
            work.wait()

    ms, _ = timer.time(run, 3, 3)
    _check_status("the row-shard run")
    gathered = sum(tokens * lin.width * world * 4 for lin in linears)
    del linears
    torch.cuda.empty_cache()
    return {"value": tokens * 1000.0 / ms, "unit": UNIT, "ms_per_step": ms, "n_gpus": world,
            "parallelism": f"u-row-shard{world}", "tokens": tokens, "scaling": "strong",
            "gathered_bytes_per_step": gathered,
            "config": "llama-3-8b 0.55 bpw, 32 layers x 7 packed linears on one 4096-token sequence; U rows split "
                      "over the ranks, fp32 output slices all-gathered in place (NCCL) on a side stream"}


def run_reference(args, rank: int) -> None:
    """The reference arm: the reference's CPU path (the oracle port) on the host cores, rank 0 only."""

    if rank != 0:
        return
    spec = WORKLOADS[args.workload]
    kind = spec["kind"]
    tokens = args.tokens or spec.get("tokens", 1)
    if kind == "step":
        base = cpu_step_baseline(tokens, steps=args.steps, warmup=args.warmup, sequences=spec.get("sequences", False))
    elif kind == "gemma":
        base = cpu_gemma_baseline(tokens, steps=args.steps, warmup=args.warmup)
    elif kind == "prefill":
        base = cpu_prefill_baseline()
    elif kind in ("single", "stacked"):
        base = cpu_linear_baseline(640, 2048, 480, tokens, layers=STACKED_LAYERS if kind == "stacked" else 1)
    elif kind == "codebook":
        base = cpu_codebook_baseline(tokens)
    else:
        raise SystemExit(f"no CPU reference path for workload {args.workload}")
    line = {
        "impl": "reference",
        "metric": spec["metric"],
        "value": base["value"],
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": base.get("steps", args.steps),
        "warmup": base.get("warmup", args.warmup),
        "ms_per_step": base["ms_per_step"],
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": spec["description"].format(layers="all", tokens=tokens), "parallelism": "cpu",
                   "cpu_model": base["cpu_model"]},
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample", "cpu_model")},
        "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=None, help="timed steps (default 20; 3 for prefill)")
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("nqb", "reference"), default="nqb")
    parser.add_argument("--workload", choices=tuple(WORKLOADS), default="decode")
    parser.add_argument("--tokens", type=int, default=None, help="tokens per step (single linear: 1 or 8)")
    parser.add_argument("--layers", type=int, default=None, help="decoder layers (default all; fewer only to profile)")
    parser.add_argument("--engine", choices=("program", "calls"), default=None,
                        help="linears workloads: one persistent program per step (default) or per-call kernels")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-extras", action="store_true", help="skip the linears / prefill / row-shard lines")
    args = parser.parse_args()
    args.warmup = max(args.warmup, 3)
    spec = WORKLOADS[args.workload]
    if args.steps is None:
        args.steps = 3 if spec["kind"] == "prefill" else 20

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    timer = Timer(device, world)
    peaks = _peak_table()

    kind = spec["kind"]
    if kind == "prefill":
        lo, hi = 0, PREFILL_TOKENS
        if args.tokens is None:
            from nanoquant_b200.sharding import token_range

            lo, hi = token_range(PREFILL_TOKENS, world, rank)
        tokens = args.tokens or (hi - lo)
    else:
        tokens = args.tokens or spec["tokens"]
    runner = _build(args.workload, device, tokens, args.layers, args.engine)
    ms_per_step, clocks = timer.time(runner.run, args.steps, args.warmup, clocks_index=local_rank)
    _check_status("the timed region")

    # end to end through the public API: the step's input from pinned host
    # memory and its output back to pinned host memory, every step
    host_in = (runner.host_input() if hasattr(runner, "host_input")
               else torch.randn(tuple(runner.input.shape)).to(runner.input.dtype)).pin_memory()
    out = runner.run()
    host_out = torch.empty(tuple(out.shape), dtype=out.dtype).pin_memory()

    def e2e_step():
        runner.input.copy_(host_in, non_blocking=True)
        host_out.copy_(runner.run(), non_blocking=True)

    e2e_ms, _ = timer.time(e2e_step, args.steps, 2)
    _check_status("the end-to-end run")

    total_tokens = tokens * world if kind != "prefill" else (args.tokens * world if args.tokens else PREFILL_TOKENS)
    value = total_tokens * 1000.0 / ms_per_step
    line: dict = {
        "metric": spec["metric"],
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": "strong" if kind == "prefill" else "weak",
        "vs_baseline": None,
        "dtype": "f16" if kind == "prefill" else "f32",
        "data": "synthetic",
        "config": {
            "workload": spec["description"].format(layers=getattr(runner, "layers", 1), tokens=tokens),
            "model": spec["model"],
            "global_batch": total_tokens,
            "tokens_per_gpu": tokens,
            "parallelism": (f"token-batches{world}" if kind == "prefill" else f"replicas{world}")
            if world > 1 else "single",
            "l2": "weights larger than the 126 MB L2 (no flush)" if kind != "single" else
                  "161 KB of weights stay in L2 across steps (config 0 is smaller than L2)",
        },
        "e2e": {
            "value": total_tokens * 1000.0 / e2e_ms,
            "unit": UNIT,
            "h2d_bytes_per_step": host_in.numel() * host_in.element_size(),
            "d2h_bytes_per_step": host_out.numel() * host_out.element_size(),
        },
        "gpu_launches": runner.launches_per_step * args.steps,
        "clocks": clocks,
    }
    if kind == "prefill" or getattr(runner, "bound", "hbm") == "tensor":
        line["roofline"] = _tensor_roofline(runner.algorithmic_flops(), ms_per_step, peaks,
                                            "all packed-linear kernels of one step per GPU (2*r*(m+n) flops per "
                                            "token and linear / step time)")
    else:
        step_bytes = runner.algorithmic_bytes()
        scope = {"step": "the whole decoder step: packed weights and scales, kv rows read, norms, lm head",
                 "gemma": "the whole decoder step: packed weights and scales, kv rows read, norms, embedding rows",
                 "linears": "the persistent decode program: every packed linear of the step in one launch",
                 "single": "one launch pair of the config-0 layer", "stacked": "the program of 1024 layers",
                 "codebook": "the program of all config-4 linears (bytes of the compact format: U words, V group "
                             "indices, tables, scales, int8 rows)"}[kind]
        line["roofline"] = _hbm_roofline(step_bytes, ms_per_step, peaks, scope)
    step_program = None
    if kind == "step" and getattr(runner.step_obj, "program", None) is not None:
        step_program = _time_step_program(runner.step_obj, args.steps, args.warmup, timer)
    del runner
    torch.cuda.empty_cache()

    if kind == "step" and not args.no_extras:
        line["step_roofline"] = line["roofline"]
        from nanoquant_b200.decode_chain import QWEN3_8B

        if step_program is not None:
            # the dominant kernel: the step's program (every layer in one launch), timed per launch
            line["roofline"] = _hbm_roofline(step_program["bytes"], step_program["ms"], peaks,
                                             "dominant kernel: the decode-step program (all 36 layers: packed "
                                             "linears, norms, q/k norm + rope, attention; bytes per launch / mean "
                                             "launch time, CUDA events around each of the timed launches)")
            line["roofline"]["launches_timed"] = step_program["launches"]
        # the packed linears alone as one program launch per step (no shell work)
        linears = ChainRunner(QWEN3_8B, device, tokens, args.layers)
        lin_ms, _ = timer.time(linears.run, args.steps, args.warmup)
        _check_status("the linears-only run")
        line["linears"] = {"value": tokens * world * 1000.0 / lin_ms, "unit": UNIT, "ms_per_step": lin_ms,
                           "algorithmic_bytes_per_step": linears.algorithmic_bytes(),
                           "roofline_frac": linears.algorithmic_bytes() / (lin_ms * 1e-3) / 1e9 / peaks["hbm"][0]}
        del linears
        torch.cuda.empty_cache()
    if not args.no_extras and kind != "prefill":
        line["prefill"] = _prefill_extra(device, timer, world, rank, peaks)
        if world > 1:
            line["row_shard"] = _row_shard_extra(device, timer, world, rank)

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        if kind == "step":
            base = cpu_step_baseline(tokens, sequences=WORKLOADS[args.workload].get("sequences", False))
        elif kind == "gemma":
            base = cpu_gemma_baseline(tokens)
        elif kind == "prefill":
            base = cpu_prefill_baseline()
        elif kind in ("single", "stacked"):
            base = cpu_linear_baseline(640, 2048, 480, tokens, layers=STACKED_LAYERS if kind == "stacked" else 1)
        elif kind == "codebook":
            base = cpu_codebook_baseline(tokens)
        else:
            base = None
        if base is not None:
            line["cpu_baseline"] = {k: base[k] for k in ("value", "unit", "cores", "kind", "sample", "cpu_model")}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
