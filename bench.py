"""Benchmark: decode tokens/s through all packed linears of a Qwen3-8B-shaped decoder (bs1).

One step = one decode token (batch 1, BASELINE config 2 shape) through the 36
layers x {q,k,v,o,gate,up,down} packed binary low-rank linears at ~1 bpw,
with the grouped QKV and gate/up calls of the reference's model shell, captured
in one CUDA graph.  Weights are random layout-v1 words (875 MB, larger than
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
UNIT = "tok/s"


def _peaks() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


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


def cpu_baseline(sample_layers: int, repeats: int) -> dict:
    """Time the CPU oracle (numpy port of PackedReferenceBackend) on ``sample_layers`` Qwen3-8B layers."""

    import numpy as np

    from nanoquant_b200.decode_chain import QWEN3_8B
    from oracle import packed_oracle as po

    rng = np.random.default_rng(0)
    shape = QWEN3_8B
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
        inputs = {proj: rng.standard_normal((1, n)).astype(np.float32) for proj, (n, _m) in shape.projections().items()}
        for proj, layer in layers.items():
            po.packed_linear(inputs[proj], layer)  # warm-up
        start = time.perf_counter()
        for _ in range(repeats):
            for proj, layer in layers.items():
                po.packed_linear(inputs[proj], layer)
        per_layer_seconds.append((time.perf_counter() - start) / repeats)
        del layers
    per_layer = statistics.median(per_layer_seconds)
    step = per_layer * shape.layers
    cores = os.cpu_count() or 1
    return {
        "value": 1.0 / step,
        "unit": UNIT,
        "cores": cores,
        "kind": "port",
        "sample": f"{sample_layers} of {shape.layers} Qwen3-8B layers x 7 projections, bs1, {repeats} reps each; "
                  f"numpy/BLAS fp32 on {cores} host threads; step time extrapolated x{shape.layers}",
        "ms_per_step": step * 1e3,
    }


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    base = cpu_baseline(sample_layers=2, repeats=max(1, args.steps))
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": base["value"],
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": base["ms_per_step"],
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "qwen3-8b packed linears, decode bs1 (36 layers x q,k,v,o,gate,up,down)",
                   "global_batch": 1, "seq_len": 1, "parallelism": "cpu"},
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=50)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("nqb", "reference"), default="nqb")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--layers", type=int, default=None,
                        help="decoder layers in the step (default: all 36); fewer only for profiling runs")
    args = parser.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist

    from nanoquant_b200.decode_chain import QWEN3_8B, DecodeChain, make_decoder_layers

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    def barrier() -> None:
        if world > 1:
            dist.barrier()

    shape = QWEN3_8B
    chain = DecodeChain(shape, make_decoder_layers(shape, device, layers=args.layers, seed=rank), device, tokens=1)
    chain.capture()
    for _ in range(args.warmup):
        chain.replay()
    torch.cuda.synchronize(device)

    stream = torch.cuda.current_stream(device)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        barrier()
        torch.cuda.synchronize(device)
        start.record(stream)
        for _ in range(args.steps):
            chain.replay()
        stop.record(stream)
        torch.cuda.synchronize(device)
        barrier()
    elapsed_ms = start.elapsed_time(stop)

    # end to end through the public API: pinned host token in, result back to host, every step
    host_in = torch.randn(1, shape.hidden).bfloat16().pin_memory()
    host_out = torch.empty(chain.graph_output.shape, dtype=torch.float32).pin_memory()
    for _ in range(2):
        chain.inputs["hidden"].copy_(host_in, non_blocking=True)
        host_out.copy_(chain.replay(), non_blocking=True)
    torch.cuda.synchronize(device)
    e_start, e_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e_start.record(stream)
    for _ in range(args.steps):
        chain.inputs["hidden"].copy_(host_in, non_blocking=True)
        host_out.copy_(chain.replay(), non_blocking=True)
    e_stop.record(stream)
    torch.cuda.synchronize(device)
    barrier()
    e2e_ms = e_start.elapsed_time(e_stop)

    if world > 1:
        times = torch.tensor([elapsed_ms, e2e_ms], device=device)
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
        elapsed_ms, e2e_ms = (float(v) for v in times.tolist())

    ms_per_step = elapsed_ms / args.steps
    value = world * 1000.0 / ms_per_step
    peak, peak_kind = _peaks()
    step_bytes = chain.algorithmic_bytes()
    achieved = step_bytes / (ms_per_step * 1e-3) / 1e9
    line = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {
            "workload": f"qwen3-8b packed linears, decode bs1 ({len(chain.blocks)} layers x q,k,v,o,gate,up,down; "
                        "grouped qkv and gate/up)",
            "model": "qwen3-8b-shape random-init packed weights ~1 bpw",
            "global_batch": world,
            "seq_len": 1,
            "parallelism": f"replicas{world}" if world > 1 else "single",
            "l2": "weights 875 MB > 126 MB L2 (no flush)",
            "cuda_graph": True,
        },
        "roofline": {
            "bound": "hbm",
            "achieved": achieved,
            "peak": peak,
            "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": None,
            "peak_kind": peak_kind,
            "scope": "all packed-linear kernels of one step (algorithmic bytes per step / step time)",
            "algorithmic_bytes_per_step": step_bytes,
        },
        "e2e": {
            "value": world * 1000.0 * args.steps / e2e_ms,
            "unit": UNIT,
            "h2d_bytes_per_step": host_in.numel() * host_in.element_size(),
            "d2h_bytes_per_step": host_out.numel() * host_out.element_size(),
        },
        "gpu_launches": chain.launches_per_step * args.steps,
        "clocks": clocks.summary(),
    }
    if rank == 0 and not args.no_cpu_baseline:
        base = cpu_baseline(sample_layers=2, repeats=3)
        line["cpu_baseline"] = {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
