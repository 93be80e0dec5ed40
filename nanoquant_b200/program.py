"""Persistent decode program: a fixed sequence of packed-linear calls in one launch.

Each op is one call of the reference's per-projection API: a single packed
linear (``RuntimeBackend.linear``) or a QKV / gate-up group
(``grouped_cuda_projection``, reference ``runtime/cuda_backend.py:286-330``),
on 1..16 tokens.  The reference replays a decode step's per-linear launches
from a CUDA graph (``runtime/torch_model.py:300-340``); here the whole
sequence is one cooperative launch of ``nqb_program_run`` (one CTA per SM,
a grid barrier after every stage, sign words streamed ahead of the barriers).
Ops run strictly in order, so an op may read an earlier op's output tensor.

Inputs and outputs are bound at construction (like a captured graph): write
new activations into the same ``x`` tensors and read the same outputs.
"""

from __future__ import annotations

import ctypes
from collections.abc import Sequence
from dataclasses import dataclass

import torch

from nanoquant_b200 import _native
from nanoquant_b200.backend import PreparedLayer
from nanoquant_b200.cuda_backend import _Sm100Payload, _check_input


@dataclass(frozen=True)
class ProgramOp:
    """One call: ``layers`` (1..3 sharing ``x``) -> one fp32 output per layer.

    With ``x2`` set, ``x`` is a gate and ``x2`` an up projection (both fp32,
    same shape) and the op's input is their gated product, formed as the op
    loads it: ``silu(x) * x2`` (SwiGLU, ``activation="silu"``) or
    ``gelu_tanh(x) * x2`` (Gemma-3's gated GELU, ``activation="gelu_tanh"``).
    The MLP's down projection (reference ``runtime/torch_model.py:395-421``,
    ``:460-505``) then shares a program with the gate/up op that produces its
    inputs.
    """

    layers: tuple[PreparedLayer, ...]
    x: torch.Tensor | None
    x2: torch.Tensor | None = None
    activation: str = "silu"
    # decoder-step extensions (``nqb_program_op_ext``): a residual-stream input
    # norm, a fused epilogue (residual add with norm statistics, or q/k head
    # norm + RoPE + KV-cache append), or an attention op (no layers, no x)
    ext: _native.ProgramOpExt | None = None

    @property
    def is_attention(self) -> bool:
        return self.ext is not None and self.ext.kind == _native.NQB_OP_ATTENTION


class DecodeProgram:
    """``ops`` compiled into one ``nqb_program`` for ``x`` tensors of ``tokens`` rows."""

    def __init__(self, ops: Sequence[ProgramOp], *, outputs: Sequence[Sequence[torch.Tensor]] | None = None) -> None:
        if not ops:
            raise ValueError("a program needs at least one op")
        linear_ops = [op for op in ops if not op.is_attention]
        if not linear_ops:
            raise ValueError("a program needs at least one linear op")
        device = linear_ops[0].x.device
        tokens = None
        self.ops = tuple(ops)
        self.outputs: list[tuple[torch.Tensor, ...]] = []
        self._keep: list[object] = []
        c_ops = (_native.ProgramOp * len(ops))()
        for index, op in enumerate(ops):
            if op.is_attention:
                if op.layers or op.x is not None:
                    raise ValueError("an attention op has no layers and no x")
                self.outputs.append(())
                self._keep.append(op.ext)
                c_ops[index].layers = None
                c_ops[index].count = 0
                c_ops[index].x = None
                c_ops[index].x_dtype = 0
                c_ops[index].y = None
                c_ops[index].x2 = None
                c_ops[index].ext = ctypes.pointer(op.ext)
                continue
            if not 1 <= len(op.layers) <= 3:
                raise ValueError("an op has 1 to 3 layers")
            payloads = tuple(layer.payload for layer in op.layers)
            if not all(isinstance(payload, _Sm100Payload) for payload in payloads):
                raise TypeError("program ops need layers prepared by CudaPackedSm100Backend")
            if op.x.device != device:
                raise ValueError("all program tensors must be on one device")
            spec = op.layers[0].spec
            _check_input(op.x, spec, device)
            if op.x2 is not None:
                if op.x.dtype != torch.float32 or op.x2.dtype != torch.float32:
                    raise ValueError("SwiGLU op inputs are fp32")
                if op.x2.shape != op.x.shape or not op.x2.is_contiguous() or op.x2.device != device:
                    raise ValueError("SwiGLU op x2 must be a contiguous tensor shaped like x on x's device")
            op_tokens = op.x.numel() // spec.in_features
            if tokens is None:
                tokens = op_tokens
            elif op_tokens != tokens:
                raise ValueError("all ops of a program take the same number of tokens")
            if outputs is not None:
                outs = tuple(outputs[index])
                for out, layer in zip(outs, op.layers, strict=True):
                    if out.dtype != torch.float32 or not out.is_contiguous() or out.device != device:
                        raise ValueError("program outputs are contiguous fp32 tensors on the program's device")
                    if out.numel() != tokens * layer.spec.out_features:
                        raise ValueError("program output has the wrong size")
            else:
                outs = tuple(
                    torch.empty((*op.x.shape[:-1], layer.spec.out_features), dtype=torch.float32, device=device)
                    for layer in op.layers
                )
            self.outputs.append(outs)
            descs = (_native.LinearDesc * len(payloads))(*(payload.desc for payload in payloads))
            ys = (ctypes.c_void_p * len(outs))(*(out.data_ptr() for out in outs))
            self._keep.extend((descs, ys, op.x, op.x2, outs, op.layers))
            c_ops[index].layers = descs
            c_ops[index].count = len(payloads)
            c_ops[index].x = op.x.data_ptr()
            if op.x2 is None:
                c_ops[index].x_dtype = _native.dtype_code(op.x.dtype)
            elif op.activation in ("silu", "gelu_tanh"):
                c_ops[index].x_dtype = _native.NQB_X_SWIGLU if op.activation == "silu" else _native.NQB_X_GEGLU
            else:
                raise ValueError(f"unknown gate activation {op.activation!r}")
            c_ops[index].y = ys
            c_ops[index].x2 = None if op.x2 is None else op.x2.data_ptr()
            c_ops[index].ext = None if op.ext is None else ctypes.pointer(op.ext)
            if op.ext is not None:
                self._keep.append(op.ext)
        if tokens is None:
            raise ValueError("a program needs at least one linear op")
        self.device = device
        self.tokens = tokens
        handle = ctypes.c_void_p(None)
        with torch.cuda.device(device):
            _native.call("nqb_program_create", c_ops, len(ops), tokens, ctypes.byref(handle))
        self._handle = handle
        needed = ctypes.c_size_t(0)
        _native.call("nqb_program_workspace_bytes", handle, ctypes.byref(needed))
        self.workspace = torch.zeros(needed.value, dtype=torch.uint8, device=device)
        ctas, cluster = ctypes.c_int32(0), ctypes.c_int32(0)
        _native.call("nqb_program_shape", handle, ctypes.byref(ctas), ctypes.byref(cluster))
        self.ctas = ctas.value
        self.cluster_size = cluster.value

    def run(self, *, dependent: bool = False) -> list[tuple[torch.Tensor, ...]]:
        """Launch the program on the current stream; returns the bound outputs.

        ``dependent=True`` launches it as a programmatic dependent of the
        preceding kernel (``nqb_program_run_dependent``): its sign words stream
        in while that kernel finishes.  For a program that follows other
        kernels; back-to-back runs of programs are faster without it.
        """

        if self._handle is None:
            raise RuntimeError("program was closed")
        _native.call(
            "nqb_program_run_dependent" if dependent else "nqb_program_run",
            self._handle,
            self.workspace.data_ptr(),
            self.workspace.numel(),
            _native.current_stream_handle(self.device),
        )
        return self.outputs

    def close(self) -> None:
        if getattr(self, "_handle", None) is not None:
            _native.call("nqb_program_destroy", self._handle)
            self._handle = None

    def __del__(self) -> None:  # pragma: no cover - interpreter shutdown order varies
        try:
            self.close()
        except Exception:
            pass


__all__ = ["DecodeProgram", "ProgramOp"]
