"""Drop-in through the reference runtime's own planner, loader and layer types.

The reference runtime (``nanoquant.runtime``) is imported from its offline
install under ``baseline/_ref`` (or from the environment).  The CPU tests run
the reference's ``plan_backends`` with ``CudaPackedSm100Backend`` in its
backend list and check that the reference's own ``PackedLayerState``,
``MixedVLayerState`` and ``ProductCodebookLayerState`` instances are adopted
field for field.  The ``gpu`` test loads layers with the reference's
``open_packed_artifact(...).load_layer`` from the fixture its writer made,
plans and prepares them with the reference's ``plan_backends`` /
``prepare_plan`` (strict, sm_100a backend only), runs them through
``PreparedBackendPlan.linear_at`` and compares with the reference's own
``PackedReferenceBackend`` on the CPU (tolerance of the reference's GPU test,
``test_runtime_cuda_backend.py:491``: rtol 2e-5, atol 2e-4).
"""

from __future__ import annotations

import dataclasses
import importlib
import sys
from pathlib import Path

import pytest
import torch

from nanoquant_b200 import CudaPackedSm100Backend, MixedVLayerState, PackedLayerState, ProductCodebookLayerState
from nanoquant_b200.cuda_backend import adopt_layer_state
from tests.fixtures import GOLDEN, load

ROOT = Path(__file__).resolve().parents[1]
REFERENCE_INSTALL = ROOT / "baseline" / "_ref"


def _reference_runtime():
    try:
        return importlib.import_module("nanoquant.runtime")
    except ImportError:
        pass
    if REFERENCE_INSTALL.is_dir():
        sys.path.insert(0, str(REFERENCE_INSTALL))
        try:
            return importlib.import_module("nanoquant.runtime")
        except ImportError:
            return None
    return None


rt = _reference_runtime()
pytestmark = pytest.mark.skipif(
    rt is None, reason="the reference runtime (nanoquant.runtime) is not importable: baseline/_ref is not installed")


def _as_reference(state):
    """The reference runtime's instance with the fields of one of this package's states."""

    classes = {PackedLayerState: rt.PackedLayerState, MixedVLayerState: rt.MixedVLayerState,
               ProductCodebookLayerState: rt.ProductCodebookLayerState}
    target = classes[type(state)]
    values = {f.name: getattr(state, f.name) for f in dataclasses.fields(target)}
    spec = values["spec"]
    values["spec"] = rt.QuantizedLinearSpec(**{f.name: getattr(spec, f.name)
                                               for f in dataclasses.fields(rt.QuantizedLinearSpec)})
    return target(**values)


def _assert_same_fields(ours, theirs) -> None:
    for field in dataclasses.fields(ours):
        a, b = getattr(ours, field.name), getattr(theirs, field.name)
        if isinstance(a, torch.Tensor):
            assert isinstance(b, torch.Tensor) and a.dtype == b.dtype and torch.equal(a, b), field.name
        elif field.name == "spec":
            for f in dataclasses.fields(a):
                assert getattr(a, f.name) == getattr(b, f.name), f.name
        else:
            assert a == b, field.name


def _packed_state() -> PackedLayerState:
    from tests.test_sharding import _state

    return _state(96, 300, 40, seed=3)


def _mixed_v_state() -> MixedVLayerState:
    from tests.test_mixed_v import mixed_v_state

    return mixed_v_state(160, 96, 70, 9, seed=2, bias=True, outliers=2)


def _codebook_state() -> ProductCodebookLayerState:
    from tests.test_host_layout import _codebook_state

    return _codebook_state(load("product_codebook"), "c4like")


@pytest.mark.parametrize("make", (_packed_state, _mixed_v_state, _codebook_state))
def test_reference_layer_states_are_adopted(make) -> None:
    ours = make()
    theirs = _as_reference(ours)
    assert type(theirs).__module__.startswith("nanoquant.runtime")
    adopted = adopt_layer_state(theirs)
    assert type(adopted) is type(ours)
    _assert_same_fields(adopted, theirs)
    assert adopt_layer_state(ours) is ours


def _specs(states: dict) -> tuple:
    return tuple(state.spec for state in states.values())


def _pretend_b200(monkeypatch) -> None:
    """The capability checks of ``supports`` see an sm_100 device (CPU planning only; nothing runs)."""

    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    monkeypatch.setattr(torch.cuda, "get_device_capability", lambda *args: (10, 0))


def test_reference_planner_selects_the_sm100_backend_strictly(monkeypatch) -> None:
    _pretend_b200(monkeypatch)
    states = {s.spec.name: s for s in (_as_reference(_packed_state()),)}
    workload = rt.WorkloadSpec("decode", "cuda", "bfloat16", 1, 1, deterministic=True)
    plan = rt.plan_backends(_specs(states), workload, (CudaPackedSm100Backend(), rt.PackedReferenceBackend()),
                            strict=True)
    assert [d.backend_name for d in plan.layers] == ["cuda-packed-sm100a"]
    assert plan.fallback_count == 0 and not plan.layers[0].fallback


def test_reference_planner_reports_our_rejection_codes() -> None:
    # no B200 in this process (CPU run) or an input dtype outside the table: the
    # strict plan fails with our stable code; a non-strict one falls back
    states = {s.spec.name: s for s in (_as_reference(_packed_state()),)}
    workload = rt.WorkloadSpec("decode", "cuda", "float64", 1, 1)
    with pytest.raises(rt.BackendPlanningError, match="cuda-packed-sm100a@1: NQ-INF-"):
        rt.plan_backends(_specs(states), workload, (CudaPackedSm100Backend(),), strict=True)
    cpu = rt.WorkloadSpec("decode", "cpu", "float32", 1, 1)
    plan = rt.plan_backends(_specs(states), cpu, (CudaPackedSm100Backend(), rt.PackedReferenceBackend()),
                            strict=False)
    dispatch = plan.layers[0]
    assert dispatch.backend_name == rt.PackedReferenceBackend().name and dispatch.fallback
    assert dispatch.rejected_backends[0].backend_name == "cuda-packed-sm100a"
    assert dispatch.rejected_backends[0].support.code.startswith("NQ-INF-")


@pytest.mark.gpu
@pytest.mark.parametrize("tokens", (1, 8))
def test_reference_loader_planner_and_linear_at_on_sm100(tokens: int) -> None:
    if not torch.cuda.is_available():
        pytest.fail("GPU test needs CUDA")
    artifact = rt.open_packed_artifact(GOLDEN / "packed_artifact")
    names = tuple(layer.spec.name for block in artifact.manifest.blocks for layer in block.layers)
    states = {name: artifact.load_layer(name) for name in names}
    assert all(type(s).__module__.startswith("nanoquant.runtime") for s in states.values())
    kind = "decode" if tokens == 1 else "prefill"
    workload = rt.WorkloadSpec(kind, "cuda", "bfloat16", 1, tokens, deterministic=True)
    backend = CudaPackedSm100Backend()
    plan = rt.plan_backends(_specs(states), workload, (backend,), strict=True)
    prepared = rt.PreparedBackendPlan(plan, rt.prepare_plan(plan, states, (backend,), "cuda"))
    reference = rt.PackedReferenceBackend()
    g = torch.Generator().manual_seed(tokens)
    for index, name in enumerate(names):
        spec = states[name].spec
        x = torch.randn(1, tokens, spec.in_features, generator=g).bfloat16()
        got = prepared.linear_at(index, x.cuda())
        again = prepared.linear_at(index, x.cuda())
        torch.cuda.synchronize()
        expected = reference.linear(x.float(), reference.prepare(states[name], "cpu"))
        assert got.dtype == torch.float32 and got.shape == (1, tokens, spec.out_features)
        assert torch.equal(got, again)  # deterministic replay
        torch.testing.assert_close(got.cpu(), expected, rtol=2e-5, atol=2e-4)
