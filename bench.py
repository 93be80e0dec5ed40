"""Benchmark: decode tokens/s through all packed linears of a Qwen3-8B-shaped decoder (bs1).

One step = one decode token (batch 1, Qwen3-8B shape) through the 36
layers x {q,k,v,o,gate,up,down} packed binary low-rank linears at ~1 bpw,
with the grouped QKV and gate/up calls of the reference's model shell, run as
one persistent decode program (a grid barrier between every stage, so the
calls stay strictly ordered); ``--engine calls`` runs the per-call kernels
captured in one CUDA graph instead.  Weights are random layout-v1 words (875 MB, larger than
the 126 MB L2, so no L2 flush is needed between steps); activations are
synthetic bf16 N(0,1).

Prints one JSON line (rank 0).  ``--impl reference`` times the CPU oracle
(the reference's packed CPU algorithm restated in numpy) on a bounded sample
of the same workload on the host cores instead.

Launch: ``python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]``;
for N > 1 under ``torch.distributed.run``: decode does not shard, so every
rank runs an independent replica ("replicas only") and ``value`` sums them.
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
PREFILL_METRIC = "prefill tok/s (Llama-3-8B shape 0.55 bpw, 8x4096 tokens); tensor TFLOP/s vs peak"
UNIT = "tok/s"


def _peak_table() -> dict[str, tuple[float, str]]:
    """HBM GB/s and sustained dense bf16 TFLOP/s: measured on this pool, else the fallback figures."""

    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm": (float(data["hbm_gbs"]), "measured"),
                "tensor": (float(data.get("bf16_tflops_sustained", data["bf16_tflops"])), "measured-sustained")}
    return {"hbm": (6650.0, "fallback"), "tensor": (1400.0, "fallback-sustained")}


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


def cpu_baseline(workload: str = "decode", repeats: int = 3) -> dict:
    """Time the CPU oracle (numpy port of PackedReferenceBackend) on a bounded sample.

    decode workloads: 2 layers of the shape at the workload's token count;
    prefill: 1 of 32 Llama-3-8B layers, 128 tokens.  The result is
    extrapolated to the full step.
    """

    import numpy as np

    from nanoquant_b200 import decode_chain
    from oracle import packed_oracle as po

    rng = np.random.default_rng(0)
    spec = WORKLOADS[workload]
    shape = getattr(decode_chain, spec["shape"])
    sample_layers, sample_tokens = (2, spec["decode_tokens"]) if spec["kind"] == "decode" else (1, 128)
    per_layer_seconds = []
    for _layer in range(sample_layers):
        layers = {}
        for proj, (n, m) in shape.projections().items():
            r = shape.rank(n, m)

            def words(rows, cols):
                raw = rng.integers(0, 2**32, size=(rows, po.word_count(cols)), dtype=np.uint64).astype(np.uint32)
                if cols % 32:
                    raw[:, -1] &= np.uint32((1 << (cols % 32)) - 1)
                return raw.view(np.int32)

            layer = po.OracleLayer(n, m, r, words(m, r), words(r, n),
                                   (np.abs(rng.standard_normal(n)) * 0.05 + 0.01).astype(np.float16).astype(np.float32),
                                   np.ones(r, np.float32),
                                   (np.abs(rng.standard_normal(m)) * 0.05 + 0.01).astype(np.float16).astype(np.float32))
            layer.prepared()  # the reference unpacks once at prepare time; not timed
            layers[proj] = layer
        inputs = {proj: rng.standard_normal((sample_tokens, n)).astype(np.float32)
                  for proj, (n, _m) in shape.projections().items()}
        for proj, layer in layers.items():
            po.packed_linear(inputs[proj], layer)  # warm-up
        start = time.perf_counter()
        for _ in range(repeats):
            for proj, layer in layers.items():
                po.packed_linear(inputs[proj], layer)
        per_layer_seconds.append((time.perf_counter() - start) / repeats)
        del layers
    per_layer = statistics.median(per_layer_seconds)
    step = per_layer * shape.layers  # one pass of `sample_tokens` tokens through every layer
    cores = os.cpu_count() or 1
    return {
        "value": sample_tokens / step,
        "unit": UNIT,
        "cores": cores,
        "kind": "port",
        "sample": f"{sample_layers} of {shape.layers} {shape.name} layers x 7 projections, {sample_tokens} token(s), "
                  f"{repeats} reps; numpy/BLAS fp32 on {cores} host threads; extrapolated to all layers",
        "ms_per_step": step * 1e3,
    }


def cpu_baseline_step(repeats: int = 1) -> dict:
    """CPU time of a full Qwen3-8B step, composed of three timed parts.

    It adds the packed linears (``cpu_baseline("decode")``, the oracle on 2
    of 36 layers), the shell math of the decoder oracle (norms, q/k norm and
    RoPE, attention over 2049 cached rows, SwiGLU) timed on 2 layers, and the
    151936 x 4096 lm head, all extrapolated to one step.
    """

    import numpy as np

    from nanoquant_b200 import decode_chain
    from oracle import decoder_oracle as do

    shape = decode_chain.QWEN3_8B
    hd, hkv, hq = shape.head_dim, shape.kv_heads, shape.q_heads
    linears = cpu_baseline("decode", repeats=1)
    rng = np.random.default_rng(0)
    caches = do.bf16(rng.standard_normal((hkv, STEP_POSITION + 1, hd)).astype(np.float32))
    h = rng.standard_normal((1, shape.hidden)).astype(np.float32)
    w = np.ones(shape.hidden, np.float32)
    qkv = rng.standard_normal((1, (hq + 2 * hkv) * hd)).astype(np.float32)
    gate = rng.standard_normal((1, shape.intermediate)).astype(np.float32)
    cos, sin = do.rope_tables(np.arange(STEP_POSITION, STEP_POSITION + 1), hd, 1e6)
    sample_layers = 2
    start = time.perf_counter()
    for _ in range(repeats * sample_layers):
        xn = do.bf16(do.rmsnorm(h, w, 1e-6))
        q = do.bf16(do.rotate(do.rmsnorm(qkv[:, : hq * hd].reshape(1, hq, hd), np.ones(hd, np.float32), 1e-6),
                              cos[:, None], sin[:, None]))
        do.attention(q, caches, caches, STEP_POSITION + 1)
        xn = do.bf16(do.rmsnorm(h + xn, w, 1e-6))
        do.bf16(gate / (1.0 + np.exp(-gate)) * gate)
    shell_layer = (time.perf_counter() - start) / (repeats * sample_layers)
    head = (0.02 * rng.standard_normal((STEP_VOCAB, shape.hidden))).astype(np.float32)
    start = time.perf_counter()
    _ = head @ h[0]
    head_s = time.perf_counter() - start
    step = linears["ms_per_step"] * 1e-3 + shell_layer * shape.layers + head_s
    cores = os.cpu_count() or 1
    return {
        "value": 1.0 / step, "unit": UNIT, "cores": cores, "kind": "port",
        "sample": f"packed linears: {linears['sample']}; shell (oracle norms, rope, attention over "
                  f"{STEP_POSITION + 1} rows, swiglu) on {sample_layers} layers and the {STEP_VOCAB} x "
                  f"{shape.hidden} lm head, extrapolated to {shape.layers} layers",
        "ms_per_step": step * 1e3,
    }


def run_reference(args, rank: int, world: int) -> None:
    """The reference arm: the reference's packed CPU algorithm (oracle port) on the host cores."""

    if rank != 0:
        return
    spec = WORKLOADS[args.workload]
    base = (cpu_baseline_step() if spec["kind"] == "step"
            else cpu_baseline(args.workload, repeats=max(1, min(args.steps, 5))))
    line = {
        "impl": "reference",
        "metric": spec["metric"],
        "value": base["value"],
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": base["ms_per_step"],
        "higher_is_better": True,
        "scaling": "weak" if spec["kind"] != "prefill" else "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": spec["description"].format(layers="all"), "model": spec["model"],
                   "parallelism": "cpu"},
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


class _StepAdapter:
    """A full decoder step (``nanoquant_b200.decoder``) behind the DecodeChain methods the timing loop uses."""

    def __init__(self, step) -> None:
        self.step_obj = step
        self.inputs = {"hidden": step.hidden_in}
        self.blocks = step.layers
        self.program = None
        self.launches_per_step = step.kernel_launches()

    def capture(self) -> None:
        self.step_obj.capture()

    def replay(self):
        return self.step_obj.replay()

    def step(self):
        return self.step_obj.step()

    def algorithmic_bytes(self) -> int:
        return self.step_obj.algorithmic_bytes()


STEP_VOCAB, STEP_POSITION = 151936, 2048


WORKLOADS = {
    "decode": {
        "kind": "decode",
        "metric": METRIC,
        "shape": "QWEN3_8B",
        "tokens_total": None,  # one token per rank (replicas)
        "decode_tokens": 1,
        "description": "qwen3-8b packed linears, decode bs1 ({layers} layers x q,k,v,o,gate,up,down; grouped qkv and gate/up)",
        "model": "qwen3-8b-shape random-init packed weights ~1 bpw",
    },
    # Qwen3-8B at batch 16 and the Gemma-3-1B decode step: extra lines beside the headline
    "decode-bs16": {
        "kind": "decode",
        "metric": "decode tok/s (bs16, Qwen3-8B shape ~1 bpw); packed-GEMV HBM GB/s vs peak",
        "shape": "QWEN3_8B",
        "tokens_total": None,
        "decode_tokens": 16,
        "description": "qwen3-8b packed linears, decode bs16 ({layers} layers x q,k,v,o,gate,up,down; grouped qkv and gate/up)",
        "model": "qwen3-8b-shape random-init packed weights ~1 bpw",
    },
    "decode-gemma1b": {
        "kind": "decode",
        "metric": "decode tok/s (bs1, Gemma-3-1B shape ~1 bpw); packed-GEMV HBM GB/s vs peak",
        "shape": "GEMMA3_1B",
        "tokens_total": None,
        "decode_tokens": 1,
        "description": "gemma-3-1b packed linears, decode bs1 ({layers} layers x q,k,v,o,gate,up,down; grouped qkv and gate/up)",
        "model": "gemma-3-1b-shape random-init packed weights ~1 bpw",
    },
    "decode-step": {
        "kind": "step",
        "metric": "decode tok/s (bs1, full Qwen3-8B-shaped step: packed linears + shell + lm head); HBM GB/s vs peak",
        "shape": "QWEN3_8B",
        "tokens_total": None,
        "decode_tokens": 1,
        "description": "qwen3-8b decode step bs1 ({layers} layers: norms, packed q/k/v/o/gate/up/down, q/k norm + "
                       "rope, attention over 2048 cached tokens, swiglu; final norm; bf16 lm head 151936 x 4096)",
        "model": "qwen3-8b-shape random-init: packed weights ~1 bpw, bf16 norms and lm head, bf16 kv cache N(0,1)",
    },
    "prefill": {
        "kind": "prefill",
        "metric": PREFILL_METRIC,
        "shape": "LLAMA3_8B_055",
        "tokens_total": 8 * 4096,  # 8 sequences x 4096 tokens, disjoint token batches per rank
        "description": "llama-3-8b packed linears, prefill 8x4096 tokens ({layers} layers x q,k,v,o,gate,up,down)",
        "model": "llama-3-8b-shape random-init packed weights 0.55 bpw",
    },
}


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=None, help="timed steps (default 50 decode, 3 prefill)")
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("nqb", "reference"), default="nqb")
    parser.add_argument("--workload", choices=tuple(WORKLOADS), default="decode",
                        help="decode: Qwen3-8B packed linears at batch 1 (the headline); prefill: Llama-3-8B 0.55 bpw, "
                             "8 x 4096 tokens")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--layers", type=int, default=None,
                        help="decoder layers in the step (default: all); fewer only for profiling runs")
    parser.add_argument("--engine", choices=("program", "calls"), default=None,
                        help="decode: one persistent program launch per step (default) or per-call kernels in a "
                             "CUDA graph")
    parser.add_argument("--tokens", type=int, default=None,
                        help="prefill tokens per GPU (default: 8*4096 / GPUs); smaller only for profiling runs")
    args = parser.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.steps is None:
        args.steps = 50 if WORKLOADS[args.workload]["kind"] != "prefill" else 3

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist

    from nanoquant_b200 import decode_chain
    from nanoquant_b200.decode_chain import DecodeChain, make_decoder_layers

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    def barrier() -> None:
        if world > 1:
            dist.barrier()

    spec = WORKLOADS[args.workload]
    shape = getattr(decode_chain, spec["shape"])
    if spec["tokens_total"] is None:
        tokens = spec["decode_tokens"]
    else:
        if spec["tokens_total"] % world:
            raise SystemExit(f"{spec['tokens_total']} tokens do not split over {world} ranks")
        tokens = spec["tokens_total"] // world
        if args.tokens is not None:
            tokens = args.tokens
    if spec["kind"] == "step":
        from nanoquant_b200.decoder import build_qwen3_step

        chain = _StepAdapter(build_qwen3_step(shape, device, vocab=STEP_VOCAB, tokens=tokens, position=STEP_POSITION,
                                              layers=args.layers))
    else:
        chain = DecodeChain(shape, make_decoder_layers(shape, device, layers=args.layers, seed=0), device,
                            tokens=tokens, engine=args.engine)
    decode = spec["kind"] in ("decode", "step")
    use_graph = decode and chain.program is None
    if use_graph:
        chain.capture()
    run_step = chain.replay if use_graph else chain.step
    for _ in range(args.warmup):
        run_step()
    torch.cuda.synchronize(device)

    stream = torch.cuda.current_stream(device)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        barrier()
        torch.cuda.synchronize(device)
        start.record(stream)
        for _ in range(args.steps):
            run_step()
        stop.record(stream)
        torch.cuda.synchronize(device)
        barrier()
    elapsed_ms = start.elapsed_time(stop)
    status = _device_status()
    if status != 0:
        raise SystemExit(f"libnqb device status {status} after the timed region (a bounded wait gave up)")

    # end to end through the public API: pinned host tokens in, result back to host, every step
    host_in = torch.randn(tokens, shape.hidden).bfloat16().pin_memory()
    last = run_step()
    host_out = torch.empty(last.shape, dtype=torch.float32).pin_memory()
    for _ in range(2):
        chain.inputs["hidden"].copy_(host_in, non_blocking=True)
        host_out.copy_(run_step(), non_blocking=True)
    torch.cuda.synchronize(device)
    e_start, e_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e_start.record(stream)
    for _ in range(args.steps):
        chain.inputs["hidden"].copy_(host_in, non_blocking=True)
        host_out.copy_(run_step(), non_blocking=True)
    e_stop.record(stream)
    torch.cuda.synchronize(device)
    barrier()
    e2e_ms = e_start.elapsed_time(e_stop)

    if world > 1:
        times = torch.tensor([elapsed_ms, e2e_ms], device=device)
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
        elapsed_ms, e2e_ms = (float(v) for v in times.tolist())

    ms_per_step = elapsed_ms / args.steps
    total_tokens = tokens * world
    value = total_tokens * 1000.0 / ms_per_step
    peaks = _peak_table()
    if decode:
        step_bytes = chain.algorithmic_bytes()
        achieved = step_bytes / (ms_per_step * 1e-3) / 1e9
        roofline = {
            "bound": "hbm", "achieved": achieved, "peak": peaks["hbm"][0], "unit": "GB/s",
            "frac": achieved / peaks["hbm"][0], "traffic": None, "peak_kind": peaks["hbm"][1],
            "scope": ("the whole decoder step: packed weights and scales, kv rows read, norms, lm head"
                      if spec["kind"] == "step" else
                      "all packed-linear kernels of one step (algorithmic bytes per step / step time)"),
            "algorithmic_bytes_per_step": step_bytes,
        }
    else:
        step_flops = chain.algorithmic_flops()
        achieved = step_flops / (ms_per_step * 1e-3) / 1e12
        roofline = {
            "bound": "tensor", "achieved": achieved, "peak": peaks["tensor"][0], "unit": "TFLOP/s",
            "frac": achieved / peaks["tensor"][0], "traffic": None, "peak_kind": peaks["tensor"][1],
            "scope": "all packed-linear kernels of one step per GPU (2*r*(m+n) flops per token and linear / step time)",
            "algorithmic_flops_per_step_per_gpu": step_flops,
        }
    line = {
        "metric": spec["metric"],
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": "weak" if decode else "strong",
        "vs_baseline": None,
        "dtype": "f32" if decode else "f16",
        "data": "synthetic",
        "config": {
            "workload": spec["description"].format(layers=len(chain.blocks)),
            "model": spec["model"],
            "global_batch": total_tokens,
            "tokens_per_gpu": tokens,
            "parallelism": (f"replicas{world}" if decode else f"token-batches{world}")
            if world > 1 else "single",
            "l2": "weights larger than the 126 MB L2 (no flush)",
            "cuda_graph": use_graph,
            "engine": ("persistent program (one cooperative launch per step)" if chain.program is not None
                       else "decode programs (4 per layer) + shell kernels in one CUDA graph" if spec["kind"] == "step"
                       else "per-call kernels"),
        },
        "roofline": roofline,
        "e2e": {
            "value": total_tokens * 1000.0 * args.steps / e2e_ms,
            "unit": UNIT,
            "h2d_bytes_per_step": host_in.numel() * host_in.element_size(),
            "d2h_bytes_per_step": host_out.numel() * host_out.element_size(),
        },
        "gpu_launches": chain.launches_per_step * args.steps,
        "clocks": clocks.summary(),
    }
    if rank == 0 and not args.no_cpu_baseline:
        base = cpu_baseline_step() if spec["kind"] == "step" else cpu_baseline(args.workload)
        line["cpu_baseline"] = {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
