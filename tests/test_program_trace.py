"""The phase-trace tool (``nanoquant_b200.program_trace``) reads the table the kernel fills.

The tool prints one column per phase of the device enum ``TracePhase`` in
``csrc/nqb_program.cu``, in its order, and one row per stage of a decoder
layer; these CPU tests keep the two sides in step (the GPU side, the trace
build itself, is exercised by running the tool; see its module docstring).
"""

from __future__ import annotations

import re
from pathlib import Path

from nanoquant_b200 import program_trace

SOURCE = Path(__file__).resolve().parents[1] / "nanoquant_b200" / "csrc" / "nqb_program.cu"


def _device_phases() -> list[str]:
    text = SOURCE.read_text()
    body = re.search(r"enum TracePhase \{(.*?)\};", text, re.S).group(1)
    names = re.findall(r"\bkTrace(\w+)", body)
    assert names[-1] == "Phases"
    return names[:-1]


def test_phase_columns_follow_the_device_enum() -> None:
    device = [re.sub(r"(?<!^)([A-Z])", r"-\1", name).lower() for name in _device_phases()]
    assert device == list(program_trace.PHASES)


def test_stage_rows_cover_a_layer() -> None:
    assert len(program_trace.STAGES) == 8  # q/k/v, o, gate/up, down: two stages each
    assert len(program_trace.STEP_STAGES) == 10  # plus the attention partials and their join
    assert program_trace.STEP_STAGES[2:4] == ("attn part", "attn join")
