"""Phase trace of the persistent decode program (profiling tool).

``python -m nanoquant_b200.program_trace [--layers 4] [--tokens 1] [--shape qwen3-8b] [--step]``

``--step`` traces the fused Qwen3 decode-step program (ten stages per layer:
q/k/v, attention partials and join, o, gate/up, down) instead of the packed
linears alone; an attention stage's work is counted in the "mma" column.

Builds the trace variant of the library (``libnqb_trace.so``: the same
kernels compiled with ``NQB_PHASE_TRACE``, whose consumer thread 0 of every
CTA records the SM cycles it spends in each phase of each stage), runs a
decoder-shaped program once after warm-up and prints, per stage of the last
layer, the mean over CTAs of every phase and the phases of the CTA that
reached the stage's grid barrier last (the stage's critical path).  Cycles are
converted at the SM clock ``--mhz`` (default: the B200's 1965 MHz boost).
"""

from __future__ import annotations

import argparse
import ctypes
import os

PHASES = ("tables", "quantise", "wait-signs", "mma", "drain", "send", "wait-quarters", "sum", "release",
          "epilogue", "grid-barrier")
STAGES = ("qkv s1", "qkv s2", "o s1", "o s2", "gate/up s1", "gate/up s2", "down s1", "down s2")
STEP_STAGES = ("qkv s1", "qkv s2", "attn part", "attn join", "o s1", "o s2", "gate/up s1", "gate/up s2", "down s1",
               "down s2")


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--layers", type=int, default=4)
    parser.add_argument("--tokens", type=int, default=1)
    parser.add_argument("--shape", choices=("qwen3-8b", "gemma-3-1b"), default="qwen3-8b")
    parser.add_argument("--mhz", type=float, default=1965.0)
    parser.add_argument("--step", action="store_true", help="trace the fused decode-step program")
    parser.add_argument("--position", type=int, default=2048, help="--step: cached tokens")
    parser.add_argument("--sequences", action="store_true",
                        help="--step: the tokens are independent sequences with their own caches")
    args = parser.parse_args()
    os.environ["NQB_LIBRARY"] = "trace"  # before the library is first loaded

    import numpy as np
    import torch

    from nanoquant_b200 import _native, decode_chain
    from nanoquant_b200.build import build

    build(trace=True)
    shape = decode_chain.QWEN3_8B if args.shape == "qwen3-8b" else decode_chain.GEMMA3_1B
    device = torch.device("cuda", 0)
    names = STAGES
    if args.step:
        from nanoquant_b200.decoder import build_qwen3_step

        step = build_qwen3_step(shape, device, vocab=1024, tokens=args.tokens, position=args.position,
                                layers=args.layers, sequences=args.sequences)
        program, run, names = step.program, step.step, STEP_STAGES
    else:
        chain = decode_chain.DecodeChain(shape, decode_chain.make_decoder_layers(shape, device, layers=args.layers),
                                         device, tokens=args.tokens, engine="program")
        program, run = chain.program, chain.step
    for _ in range(3):
        run()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    run()
    stop.record()
    torch.cuda.synchronize()
    per_layer = len(names)
    stages = per_layer * args.layers
    buf = (ctypes.c_int64 * (program.ctas * stages * len(PHASES)))()
    _native.call("nqb_program_trace", program._handle, buf, len(buf))
    cycles = np.frombuffer(buf, dtype=np.int64).reshape(program.ctas, stages, len(PHASES))
    us = cycles / args.mhz
    print(f"{shape.name}, {args.layers} layers, {args.tokens} token(s): {program.ctas} CTAs, "
          f"{start.elapsed_time(stop) * 1e3:.1f} us per {'step' if args.step else 'program'} run (trace build)")
    print("per stage of the last layer: mean over CTAs | CTA with the longest time before the grid barrier (us)")
    print(f"{'stage':12s} " + " ".join(f"{p:>9s}" for p in PHASES))
    for g in range(stages - per_layer, stages):
        p = us[:, g, :]
        pre = p[:, :-1].sum(axis=1)
        worst = int(pre.argmax())
        print(f"{names[g % per_layer]:12s} " + " ".join(f"{v:9.2f}" for v in p.mean(axis=0)))
        print(f"{'  critical':12s} " + " ".join(f"{v:9.2f}" for v in p[worst]) + f"   (CTA {worst}, {pre[worst]:.2f})")


if __name__ == "__main__":
    main()
