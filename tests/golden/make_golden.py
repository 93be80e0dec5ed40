"""Generate the golden fixtures in ``tests/golden/`` from the NanoQuant reference.

Run in a checkout that has the reference source tree::

    PYTHONPATH=<reference>/src python tests/golden/make_golden.py <reference>/src

It imports the reference's own runtime (``nanoquant.runtime``) and records, for
seeded inputs, what the reference computes: layout-v1 words, product-codebook
and mixed-V decodes, ``PackedReferenceBackend.linear`` outputs on fp32
input (``src/nanoquant/runtime/reference.py:184-235``), and a small packed
artifact written by the reference's artifact writer.  The fixtures are
small ``.npz`` files; tests and the oracle read them and never need the
reference itself.  Half-precision tensors are stored as their raw 16-bit
patterns with a ``<name>__dtype`` tag.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _store(value: torch.Tensor | None, name: str, out: dict) -> None:
    if value is None:
        return
    value = value.detach().cpu().contiguous()
    if value.dtype in (torch.float16, torch.bfloat16):
        out[name] = value.view(torch.int16).numpy()
        out[name + "__dtype"] = np.array(str(value.dtype).removeprefix("torch."))
    else:
        out[name] = value.numpy()
        out[name + "__dtype"] = np.array(str(value.dtype).removeprefix("torch."))


def _signs(generator: torch.Generator, rows: int, columns: int) -> torch.Tensor:
    return torch.where(torch.rand(rows, columns, generator=generator) > 0.5, 1.0, -1.0)


def _packed_case(rt, name, *, n, m, r, tokens, seed, scale_dtype=torch.float32, outlier_dtype=None,
                 outlier_count=0, bias=False, patch=False, input_dtype=torch.bfloat16, baseline_scales=False):
    g = torch.Generator().manual_seed(seed)
    outlier_count = outlier_count if outlier_dtype is not None else 0
    spec = rt.QuantizedLinearSpec(
        "blocks.0.linear", "nanoquant-v1", n, m, r, "float32", str(scale_dtype).removeprefix("torch."),
        outlier_count=outlier_count,
        outlier_value_dtype=str(outlier_dtype).removeprefix("torch.") if outlier_count else None,
        has_outlier_scales=outlier_dtype is torch.int8 and outlier_count > 0,
        has_bias=bias,
        patch_rank=2 if patch else 0,
        patch_value_dtype=str(scale_dtype).removeprefix("torch.") if patch else None,
    )
    left = _signs(g, m, r)
    right = _signs(g, r, n)
    if baseline_scales:
        pre = (torch.randn(n, generator=g).abs() * 0.05 + 0.01).to(scale_dtype)
        mid = torch.ones(r).to(scale_dtype)
        post = (torch.randn(m, generator=g).abs() * 0.05 + 0.01).to(scale_dtype)
    else:
        pre = torch.randn(n, generator=g).to(scale_dtype)
        mid = torch.randn(r, generator=g).to(scale_dtype)
        post = torch.randn(m, generator=g).to(scale_dtype)
    indices = None
    values = None
    scales = None
    if outlier_count:
        indices = torch.sort(torch.randperm(n, generator=g)[:outlier_count]).values.to(torch.int64)
        pre[indices] = 0
        if outlier_dtype is torch.int8:
            values = torch.randint(-8, 8, (m, outlier_count), generator=g, dtype=torch.int8)
            scales = torch.linspace(0.125, 0.25, outlier_count).to(scale_dtype)
        else:
            values = torch.randn(m, outlier_count, generator=g).to(outlier_dtype)
    logical = rt.LogicalLayerState(
        spec, left, right, pre, mid, post,
        bias=torch.randn(m, generator=g).to(scale_dtype) if bias else None,
        outlier_indices=indices,
        outlier_values=values,
        outlier_scales=scales,
        patch_left=torch.randn(m, 2, generator=g).to(scale_dtype) if patch else None,
        patch_right=torch.randn(2, n, generator=g).to(scale_dtype) if patch else None,
    )
    packed = rt.pack_logical_layer(logical)
    x = torch.randn(*tokens, n, generator=g).to(input_dtype)
    backend = rt.PackedReferenceBackend()
    y = backend.linear(x.float(), backend.prepare(packed, "cpu"))
    out: dict = {"in_features": np.array(n), "out_features": np.array(m), "rank": np.array(r)}
    for field in ("left_words", "right_words", "scale_pre", "scale_mid", "scale_post", "bias",
                  "outlier_indices", "outlier_values", "outlier_scales", "patch_left", "patch_right"):
        _store(getattr(packed, field), field, out)
    _store(x, "x", out)
    _store(y, "y", out)
    np.savez_compressed(HERE / f"linear_{name}.npz", **out)


def make_packing(rt) -> None:
    out: dict = {}
    g = torch.Generator().manual_seed(5)
    for columns in (1, 31, 32, 33, 65, 128):
        signs = _signs(g, 3, columns)
        out[f"signs_{columns}"] = signs.numpy()
        out[f"words_{columns}"] = rt.pack_sign_matrix(signs).numpy()
        pattern = torch.where(torch.arange(3 * columns).reshape(3, columns) % 3 == 0, -1.0, 1.0)
        out[f"pattern_{columns}"] = pattern.numpy()
        out[f"pattern_words_{columns}"] = rt.pack_sign_matrix(pattern).numpy()
    kat = torch.ones(2, 32)
    kat[0, (0, 1, 31)] = -1
    kat[1] = -1
    out["kat_signs"] = kat.numpy()
    out["kat_words"] = rt.pack_sign_matrix(kat).numpy()
    big = _signs(g, 64, 1000)
    out["big_signs"] = big.numpy()
    out["big_words"] = rt.pack_sign_matrix(big).numpy()
    np.savez_compressed(HERE / "packing.npz", **out)


def make_linear(rt) -> None:
    # reference CUDA-backend fixture shape (tests/unit/test_runtime_cuda_backend.py:60-120): 35 -> 17, rank 33
    for outlier in (None, torch.float16, torch.bfloat16, torch.float32, torch.int8):
        tag = "none" if outlier is None else str(outlier).removeprefix("torch.")
        for tokens, ttag in (((1,), "t1"), ((2, 3), "t2x3")):
            _packed_case(rt, f"fixture_{tag}_{ttag}", n=35, m=17, r=33, tokens=tokens, seed=19,
                         scale_dtype=torch.bfloat16, outlier_dtype=outlier, outlier_count=2, bias=True)
    _packed_case(rt, "fixture_patch", n=35, m=17, r=33, tokens=(2,), seed=21, scale_dtype=torch.float32,
                 bias=True, patch=True, input_dtype=torch.float32)
    _packed_case(rt, "fixture_salient33", n=35, m=17, r=33, tokens=(2,), seed=22, scale_dtype=torch.bfloat16,
                 outlier_dtype=torch.float32, outlier_count=33, input_dtype=torch.float32)
    for index, (xdt, sdt) in enumerate(((torch.float16, torch.float16), (torch.float32, torch.bfloat16),
                                        (torch.bfloat16, torch.float32))):
        _packed_case(rt, f"dtypes_{index}", n=35, m=17, r=33, tokens=(2,), seed=40 + index, scale_dtype=sdt,
                     outlier_dtype=sdt, outlier_count=2, input_dtype=xdt)
    # llama.cpp test-backend-ops shapes (evidence dirty.patch:2704-2730): (in, rank, out, cols, salient)
    _packed_case(rt, "ggml_32_16_24", n=32, r=16, m=24, tokens=(1,), seed=31)
    _packed_case(rt, "ggml_33_17_25", n=33, r=17, m=25, tokens=(1,), seed=32, outlier_dtype=torch.float32,
                 outlier_count=3)
    _packed_case(rt, "ggml_64_32_48_i8", n=64, r=32, m=48, tokens=(4,), seed=33, outlier_dtype=torch.int8,
                 outlier_count=4)
    _packed_case(rt, "ggml_64_32_48_f16", n=64, r=32, m=48, tokens=(8,), seed=34, outlier_dtype=torch.float16,
                 outlier_count=2)
    _packed_case(rt, "ggml_96_64_64_f16", n=96, r=64, m=64, tokens=(8,), seed=35, outlier_dtype=torch.float16,
                 outlier_count=7)
    # Gemma-3-270m MLP up-proj, 640 -> 2048, rank 480, fp16 scales, mid = 1
    for tokens in (1, 8):
        _packed_case(rt, f"c0_t{tokens}", n=640, m=2048, r=480, tokens=(tokens,), seed=0,
                     scale_dtype=torch.float16, baseline_scales=True)


def make_grouped(rt) -> None:
    # reference grouped fixture (test_runtime_cuda_backend.py:152-224)
    for index, (rank, out_features) in enumerate(((32, 24), (40, 16), (48, 32))):
        g = torch.Generator().manual_seed(700 + index)
        n = 64
        spec = rt.QuantizedLinearSpec(f"blocks.0.self_attn.group_{index}", "nanoquant-v1", n, out_features, rank,
                                      "float32", "bfloat16", outlier_count=2, outlier_value_dtype="bfloat16")
        pre = torch.randn(n, generator=g).bfloat16()
        idx = torch.tensor((1, 7), dtype=torch.int64)
        pre[idx] = 0
        logical = rt.LogicalLayerState(
            spec, _signs(g, out_features, rank), _signs(g, rank, n), pre,
            torch.randn(rank, generator=g).bfloat16(), torch.randn(out_features, generator=g).bfloat16(),
            outlier_indices=idx, outlier_values=torch.randn(out_features, 2, generator=g).bfloat16())
        packed = rt.pack_logical_layer(logical)
        x = torch.randn(3, n, generator=torch.Generator().manual_seed(99))
        backend = rt.PackedReferenceBackend()
        y = backend.linear(x, backend.prepare(packed, "cpu"))
        out: dict = {"in_features": np.array(n), "out_features": np.array(out_features), "rank": np.array(rank)}
        for field in ("left_words", "right_words", "scale_pre", "scale_mid", "scale_post", "outlier_indices",
                      "outlier_values"):
            _store(getattr(packed, field), field, out)
        _store(x, "x", out)
        _store(y, "y", out)
        np.savez_compressed(HERE / f"grouped_{index}.npz", **out)


def make_product_codebook(rt) -> None:
    out: dict = {}
    indices = ((torch.arange(15).reshape(3, 5) * 7919) % 65536).to(torch.int32)
    out["kat_indices"] = indices.numpy()
    out["kat_payload"] = rt.pack_product_codebook_indices(indices).numpy()
    g = torch.Generator().manual_seed(4)
    for tag, (n, m, r, free_rows, transposed) in {
        "small": (35, 3, 7, 2, False),
        "small_t": (35, 3, 7, 2, True),
        "c4like": (96, 64, 40, 1, False),
    }.items():
        spec = rt.QuantizedLinearSpec(f"blocks.0.{tag}", "nanoquant-v1", n, m, r, "float32", "float16")
        factor_out = n if transposed else m
        factor_in = m if transposed else n
        per_row = (factor_in + 31) // 32
        table = _signs(g, 256, 16)
        first = rt.pack_product_half_table(table)
        second = first.clone()
        records = torch.randint(0, 65536, (r - free_rows, per_row), generator=g, dtype=torch.int32)
        tail = factor_in % 32
        if tail:
            # the last word of each coded row must keep its padding bits zero: use record 0
            # after forcing table entry 0 to +1 everywhere
            records[:, -1] = 0
        table[0] = 1
        first = rt.pack_product_half_table(table)
        second = first.clone()
        free = rt.pack_sign_matrix(_signs(g, free_rows, factor_in))
        state = rt.ProductCodebookLayerState(
            spec, rt.PRODUCT_CODEBOOK_FORMAT_VERSION, transposed, free_rows,
            rt.pack_sign_matrix(_signs(g, factor_out, r)), free,
            rt.pack_product_codebook_indices(records), first, second,
            (torch.randn(factor_in, generator=g).abs() * 0.05 + 0.01).half(),
            torch.ones(r).half(),
            (torch.randn(factor_out, generator=g).abs() * 0.05 + 0.01).half(),
        )
        packed = state.to_packed()
        x = torch.randn(2, n, generator=g).bfloat16()
        backend = rt.PackedReferenceBackend()
        y = backend.linear(x.float(), backend.prepare(packed, "cpu"))
        for field in ("factor_left_words", "factor_right_free_words", "factor_right_coded_payload",
                      "first_half_words", "second_half_words", "factor_scale_pre", "factor_scale_mid",
                      "factor_scale_post"):
            _store(getattr(state, field), f"{tag}_{field}", out)
        out[f"{tag}_shape"] = np.array((n, m, r, free_rows, int(transposed)))
        _store(packed.left_words, f"{tag}_left_words", out)
        _store(packed.right_words, f"{tag}_right_words", out)
        _store(packed.scale_pre, f"{tag}_scale_pre", out)
        _store(packed.scale_post, f"{tag}_scale_post", out)
        _store(x, f"{tag}_x", out)
        _store(y, f"{tag}_y", out)
    np.savez_compressed(HERE / "product_codebook.npz", **out)


def make_mixed_v(rt) -> None:
    indices = (torch.arange(34, dtype=torch.int32).reshape(2, 17) * 29) % 1024
    pairs = (torch.arange(34, dtype=torch.int32).reshape(2, 17) * 13) % 496
    payload = rt.pack_mixed_v_records(indices, pairs)
    g = torch.Generator().manual_seed(9)
    codebook = torch.randint(0, 2**32, (1024,), generator=g, dtype=torch.int64).to(torch.int32)
    free = rt.pack_sign_matrix(_signs(g, 2, 64))
    rec_idx = torch.randint(0, 1024, (5, 2), generator=g, dtype=torch.int32)
    rec_pair = torch.randint(0, 496, (5, 2), generator=g, dtype=torch.int32)
    decoded = rt.decode_mixed_v_right_words(free, rt.pack_mixed_v_records(rec_idx, rec_pair), codebook,
                                            rank=7, in_features=64)
    np.savez_compressed(
        HERE / "mixed_v.npz",
        kat_indices=indices.numpy(), kat_pairs=pairs.numpy(), kat_payload=payload.numpy(),
        codebook=codebook.numpy(), free=free.numpy(), rec_idx=rec_idx.numpy(), rec_pair=rec_pair.numpy(),
        payload=rt.pack_mixed_v_records(rec_idx, rec_pair).numpy(), decoded=decoded.numpy(),
    )


def make_packed_artifact(rt) -> None:
    """A two-block packed artifact written by the reference's own writer
    (``packed_artifact.py:306-372``) plus what its ``load_layer`` returns."""

    import shutil

    def layer(name, n, m, r, seed, scale_dtype, *, outliers=0, patch=False):
        g = torch.Generator().manual_seed(seed)
        spec = rt.QuantizedLinearSpec(
            name, "nanoquant-v1", n, m, r, "float32", str(scale_dtype).removeprefix("torch."),
            outlier_count=outliers, outlier_value_dtype="int8" if outliers else None,
            has_outlier_scales=bool(outliers), has_bias=True,
            patch_rank=2 if patch else 0, patch_value_dtype="float32" if patch else None,
        )
        pre = (torch.randn(n, generator=g).abs() * 0.05 + 0.01).to(scale_dtype)
        idx = None
        if outliers:
            idx = torch.sort(torch.randperm(n, generator=g)[:outliers]).values.to(torch.int64)
            pre[idx] = 0
        return rt.pack_logical_layer(rt.LogicalLayerState(
            spec, _signs(g, m, r), _signs(g, r, n), pre,
            (torch.randn(r, generator=g).abs() + 0.5).to(scale_dtype),
            (torch.randn(m, generator=g).abs() * 0.05 + 0.01).to(scale_dtype),
            bias=torch.randn(m, generator=g).to(scale_dtype),
            outlier_indices=idx,
            outlier_values=torch.randint(-127, 128, (m, outliers), generator=g, dtype=torch.int8) if outliers else None,
            outlier_scales=torch.full((outliers,), 0.002).to(scale_dtype) if outliers else None,
            patch_left=torch.randn(m, 2, generator=g) if patch else None,
            patch_right=torch.randn(2, n, generator=g) if patch else None,
        ))

    blocks = {
        0: [layer("blocks.0.self_attn.q_proj", 35, 3, 33, 61, torch.float32, outliers=2),
            layer("blocks.0.mlp.up_proj", 97, 50, 40, 62, torch.float16)],
        1: [layer("blocks.1.self_attn.o_proj", 64, 17, 9, 63, torch.bfloat16, patch=True)],
    }
    names = [state.spec.name for states in blocks.values() for state in states]
    root = HERE / "packed_artifact"
    if root.exists():
        shutil.rmtree(root)
    metadata = rt.RuntimeModelMetadata("fixture/model", "revision", "fixture", "config", "tokenizer")
    artifact = rt.write_packed_artifact(root, metadata, "0" * 64, blocks)
    out: dict = {}
    for name in names:
        loaded = artifact.load_layer(name)
        for field in ("left_words", "right_words", "scale_pre", "scale_mid", "scale_post", "bias",
                      "outlier_indices", "outlier_values", "outlier_scales", "patch_left", "patch_right"):
            _store(getattr(loaded, field), f"{name}:{field}", out)
    np.savez_compressed(HERE / "packed_artifact_layers.npz", **out)


def main() -> None:
    if len(sys.argv) > 1:
        sys.path.insert(0, sys.argv[1])
    import nanoquant.runtime as rt

    torch.manual_seed(0)
    make_packing(rt)
    make_linear(rt)
    make_grouped(rt)
    make_product_codebook(rt)
    make_mixed_v(rt)
    make_packed_artifact(rt)
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
