"""Loaders for the golden fixtures in ``tests/golden`` (made by ``tests/golden/make_golden.py``)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"

_TORCH = {
    "float16": torch.float16,
    "bfloat16": torch.bfloat16,
    "float32": torch.float32,
    "int8": torch.int8,
    "int16": torch.int16,
    "int32": torch.int32,
    "int64": torch.int64,
}


def load(name: str) -> dict[str, object]:
    """Return the arrays of ``golden/<name>.npz``; tagged entries become torch tensors."""

    with np.load(GOLDEN / f"{name}.npz") as data:
        raw = {key: data[key] for key in data.files}
    out: dict[str, object] = {}
    for key, value in raw.items():
        if key.endswith("__dtype"):
            continue
        tag = raw.get(key + "__dtype")
        if tag is None:
            out[key] = value
            continue
        dtype = _TORCH[str(tag)]
        if dtype in (torch.float16, torch.bfloat16):
            out[key] = torch.from_numpy(np.ascontiguousarray(value)).view(dtype)
        else:
            out[key] = torch.from_numpy(np.ascontiguousarray(value)).to(dtype)
    return out


def linear_names() -> list[str]:
    return sorted(path.stem for path in GOLDEN.glob("linear_*.npz"))


def as_numpy_f32(value: torch.Tensor | None) -> np.ndarray | None:
    if value is None:
        return None
    if value.dtype in (torch.float16, torch.bfloat16):
        return value.float().numpy()
    return value.numpy()
