"""The C-ABI library loads, exports every declared symbol, and validates arguments (CPU only).

No call here reaches a CUDA API: every case is rejected by host-side validation.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

from nanoquant_b200 import CudaPackedSm100Backend, QuantizedLinearSpec, WorkloadSpec, _native

HEADER = Path(__file__).resolve().parents[1] / "include" / "nqb.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(nqb_[a-z_0-9]+)\s*\(", text)))


def test_header_declares_the_bound_functions() -> None:
    assert set(declared_functions()) == set(_native.SIGNATURES)


def test_library_exports_every_declared_symbol() -> None:
    lib = _native.library()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert lib.nqb_abi_version() == 5


def _desc() -> _native.LinearDesc:
    desc = _native.LinearDesc()
    desc.in_features, desc.out_features, desc.rank = 64, 32, 16
    # fake, never-dereferenced device addresses (validation only)
    desc.left_words = desc.right_words = 0x10000
    desc.scale_pre = desc.scale_mid = desc.scale_post = 0x20000
    desc.scale_dtype = _native.NQB_F16
    return desc


def _status(fn: str, *args) -> tuple[int, str]:
    lib = _native.library()
    status = getattr(lib, fn)(*args)
    return status, lib.nqb_last_error().decode()


def test_workspace_size_is_reported_without_a_device() -> None:
    size = ctypes.c_size_t(0)
    status, _ = _status("nqb_linear_workspace_bytes", ctypes.byref(_desc()), 8, ctypes.byref(size))
    assert status == _native.NQB_OK
    assert size.value >= 8 * 16 * 4 and size.value % 256 == 0


def test_workspace_holds_the_patch_latent() -> None:
    plain, patched = ctypes.c_size_t(0), ctypes.c_size_t(0)
    desc = _desc()
    assert _status("nqb_linear_workspace_bytes", ctypes.byref(desc), 8, ctypes.byref(plain))[0] == _native.NQB_OK
    desc.patch_rank, desc.patch_left, desc.patch_right, desc.patch_dtype = 24, 0x80000, 0x90000, _native.NQB_BF16
    assert _status("nqb_linear_workspace_bytes", ctypes.byref(desc), 8, ctypes.byref(patched))[0] == _native.NQB_OK
    assert patched.value - plain.value == 768  # 8 tokens x 24 fp32, rounded to 256 bytes


def test_ctypes_structs_match_the_header(tmp_path) -> None:
    """Every field of the ctypes mirrors sits at the C compiler's offset for ``include/nqb.h``."""

    import shutil
    import subprocess

    compiler = shutil.which("gcc") or shutil.which("cc")
    if compiler is None:
        pytest.skip("no C compiler")
    structs = {"nqb_linear_desc": _native.LinearDesc, "nqb_program_op": _native.ProgramOp,
               "nqb_program_op_ext": _native.ProgramOpExt}
    lines = ["#include <stddef.h>", "#include <stdio.h>", '#include "nqb.h"', "int main(void) {"]
    for cname, cls in structs.items():
        lines.append(f'  printf("{cname} sizeof %zu\\n", sizeof({cname}));')
        for field, _ in cls._fields_:
            lines.append(f'  printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines += ["  return 0;", "}"]
    source = tmp_path / "layout.c"
    source.write_text("\n".join(lines) + "\n")
    include = Path(__file__).resolve().parents[1] / "include"
    exe = tmp_path / "layout"
    subprocess.run([compiler, "-std=c11", f"-I{include}", str(source), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    seen = {}
    for line in filter(None, out):
        cname, field, value = line.split()
        seen[(cname, field)] = int(value)
    for cname, cls in structs.items():
        assert seen[(cname, "sizeof")] == ctypes.sizeof(cls), cname
        for field, _ in cls._fields_:
            assert seen[(cname, field)] == getattr(cls, field).offset, (cname, field)


@pytest.mark.parametrize(
    ("mutate", "code", "message"),
    [
        (lambda d: setattr(d, "rank", 0), _native.NQB_ERR_INVALID_ARGUMENT, "must be positive"),
        (lambda d: setattr(d, "left_words", None), _native.NQB_ERR_INVALID_ARGUMENT, "left_words is NULL"),
        (lambda d: setattr(d, "right_words", None), _native.NQB_ERR_INVALID_ARGUMENT, "right_words is NULL"),
        (lambda d: setattr(d, "left_words", 0x10002), _native.NQB_ERR_ALIGNMENT, "4-byte aligned"),
        (lambda d: setattr(d, "scale_dtype", _native.NQB_I8), _native.NQB_ERR_DTYPE, "scale dtype"),
        (lambda d: (setattr(d, "outlier_count", 2), setattr(d, "outlier_indices", 0x30000),
                    setattr(d, "outlier_values", 0x30000), setattr(d, "outlier_value_dtype", _native.NQB_I8)),
         _native.NQB_ERR_INVALID_ARGUMENT, "int8 values"),
        (lambda d: setattr(d, "outlier_count", 65), _native.NQB_ERR_INVALID_ARGUMENT, "outlier count"),
        (lambda d: (setattr(d, "codebook_payload", 0x40000)), _native.NQB_ERR_INVALID_ARGUMENT, "not both"),
        (lambda d: setattr(d, "overlay_rows", 33), _native.NQB_ERR_INVALID_ARGUMENT, "overlay row count"),
        (lambda d: setattr(d, "patch_rank", -1), _native.NQB_ERR_INVALID_ARGUMENT, "patch rank"),
        (lambda d: setattr(d, "patch_rank", 4), _native.NQB_ERR_INVALID_ARGUMENT, "patch factors are NULL"),
        (lambda d: (setattr(d, "patch_rank", 4), setattr(d, "patch_left", 0x80000), setattr(d, "patch_right", 0x80000),
                    setattr(d, "patch_dtype", _native.NQB_I8)), _native.NQB_ERR_DTYPE, "patch dtype"),
    ],
)
def test_descriptor_validation(mutate, code: int, message: str) -> None:
    desc = _desc()
    mutate(desc)
    status, text = _status("nqb_linear", ctypes.byref(desc), 0x50000, _native.NQB_BF16, 1, 0x60000, 0x70000,
                           1 << 20, None)
    assert status == code
    assert message in text


def test_input_and_workspace_validation() -> None:
    desc = _desc()
    status, text = _status("nqb_linear", ctypes.byref(desc), None, _native.NQB_BF16, 1, 0x60000, 0x70000, 1 << 20, None)
    assert status == _native.NQB_ERR_INVALID_ARGUMENT and "input x" in text
    status, text = _status("nqb_linear", ctypes.byref(desc), 0x50000, _native.NQB_I8, 1, 0x60000, 0x70000, 1 << 20, None)
    assert status == _native.NQB_ERR_DTYPE
    status, text = _status("nqb_linear", ctypes.byref(desc), 0x50000, _native.NQB_BF16, 0, 0x60000, 0x70000, 1 << 20, None)
    assert status == _native.NQB_ERR_INVALID_ARGUMENT
    status, text = _status("nqb_linear", ctypes.byref(desc), 0x50000, _native.NQB_BF16, 4, 0x60000, 0x70000, 16, None)
    assert status == _native.NQB_ERR_WORKSPACE and "workspace" in text


def test_tiles_only_layers_validate_and_refuse_the_generic_path() -> None:
    desc = _desc()
    desc.left_words = desc.right_words = None
    size = ctypes.c_size_t(0)
    status, text = _status("nqb_linear_workspace_bytes", ctypes.byref(desc), 8, ctypes.byref(size))
    assert status == _native.NQB_ERR_INVALID_ARGUMENT and "needs both tile copies" in text
    desc.left_tiles, desc.right_tiles = 0x90000, 0xA0000  # fake, never dereferenced
    status, _ = _status("nqb_linear_workspace_bytes", ctypes.byref(desc), 8, ctypes.byref(size))
    assert status == _native.NQB_OK
    tokens = (1 << 22) + 1  # past the prefill path's token limit: only the generic kernels take it
    path = ctypes.c_int32(-1)
    status, _ = _status("nqb_linear_path", ctypes.byref(desc), 1, _native.NQB_BF16, tokens, ctypes.byref(path))
    assert status == _native.NQB_OK and path.value == _native.NQB_PATH_GENERIC
    # refused on the host before any launch
    status, text = _status("nqb_linear", ctypes.byref(desc), 0x50000, _native.NQB_BF16, tokens, 0x60000, 0x100000,
                           1 << 40, None)
    assert status == _native.NQB_ERR_UNSUPPORTED and "generic path" in text


def test_grouped_rejects_mismatched_inputs() -> None:
    descs = (_native.LinearDesc * 2)(_desc(), _desc())
    descs[1].in_features = 65
    outs = (ctypes.c_void_p * 2)(0x60000, 0x61000)
    status, text = _status("nqb_grouped_linear", descs, 2, 0x50000, _native.NQB_BF16, 1, outs, 0x70000, 1 << 20, None)
    assert status == _native.NQB_ERR_INVALID_ARGUMENT and "share in_features" in text
    status, _ = _status("nqb_grouped_linear", descs, 4, 0x50000, _native.NQB_BF16, 1, outs, 0x70000, 1 << 20, None)
    assert status == _native.NQB_ERR_INVALID_ARGUMENT


def test_backend_capabilities_and_rejection_codes() -> None:
    backend = CudaPackedSm100Backend()
    caps = backend.capabilities()
    assert caps.device_types == ("cuda",)
    assert "int8" in caps.outlier_value_dtypes
    spec = QuantizedLinearSpec("blocks.0.q", "nanoquant-v1", 64, 32, 16, "float32", "float16")
    cpu = backend.supports(spec, WorkloadSpec("decode", "cpu", "bfloat16", 1, 1))
    assert (cpu.supported, cpu.code) == (False, "NQ-INF-DEVICE")
    fmt = backend.supports(
        QuantizedLinearSpec("blocks.0.q", "other", 64, 32, 16, "float32", "float16"),
        WorkloadSpec("decode", "cuda", "bfloat16", 1, 1),
    )
    assert fmt.code == "NQ-INF-FORMAT"
    if not torch.cuda.is_available():
        missing = backend.supports(spec, WorkloadSpec("decode", "cuda", "bfloat16", 1, 1))
        assert missing.code == "NQ-INF-DEVICE-UNAVAILABLE"


def test_prepare_refuses_cpu_device() -> None:
    from tests.fixtures import load
    from nanoquant_b200 import PACKED_LAYOUT_VERSION, PackedLayerState

    case = load("linear_ggml_32_16_24")
    spec = QuantizedLinearSpec("blocks.0.l", "nanoquant-v1", 32, 24, 16, "float32", "float32")
    state = PackedLayerState(spec, PACKED_LAYOUT_VERSION, case["left_words"], case["right_words"],
                             case["scale_pre"], case["scale_mid"], case["scale_post"])
    with pytest.raises(ValueError, match="requires a CUDA device"):
        CudaPackedSm100Backend().prepare(state, "cpu")


@pytest.mark.parametrize(
    "q, k, v, out, workspace",
    [
        (0x10004, 0x20000, 0x30000, 0x40000, 0x50000),  # q 4-byte aligned, head_dim 128 needs 8
        (0x10000, 0x20008, 0x30000, 0x40000, 0x50000),  # k cache 8-byte aligned, needs 16
        (0x10000, 0x20000, 0x30008, 0x40000, 0x50000),  # v cache
        (0x10000, 0x20000, 0x30000, 0x40002, 0x50000),  # out
        (0x10000, 0x20000, 0x30000, 0x40000, 0x50004),  # workspace
    ],
)
def test_decode_attention_rejects_misaligned_operands(q, k, v, out, workspace) -> None:
    status, message = _status("nqb_decode_attention", q, k, v, 4096, 2049, 1, 32, 8, 128, out, workspace,
                              1 << 24, None)
    assert status == _native.NQB_ERR_ALIGNMENT, message
    assert "alignment" in message


def test_workspace_reset_needs_the_counter_region() -> None:
    status, message = _status("nqb_workspace_reset", 0x10000, 1024, None)
    assert status == _native.NQB_ERR_WORKSPACE, message
    status, message = _status("nqb_workspace_reset", None, 1 << 20, None)
    assert status == _native.NQB_ERR_WORKSPACE, message


def test_debug_barrier_skew_rejects_a_null_program() -> None:
    status, _ = _status("nqb_program_debug_barrier_skew", None, 1)
    assert status == _native.NQB_ERR_INVALID_ARGUMENT
