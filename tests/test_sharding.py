"""Multi-GPU partitions of the packed linear, checked on CPU with the oracle.

The host-side logic of the token-batch and U-row-shard partitions
(``nanoquant_b200.sharding``) runs here under ``torch.distributed`` with the
``gloo`` backend and two ranks; the per-rank linear is the oracle (the CPU
restatement of the reference's packed path), so the tests check that the
partition, the row slicing of every per-row tensor and the all-gather put
each output element where the unsharded layer computes it.
"""

from __future__ import annotations

import os
import socket
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nanoquant_b200 import (
    LogicalLayerState,
    OutlierRowOverlay,
    OverlaidLayerState,
    PackedLayerState,
    QuantizedLinearSpec,
    pack_logical_layer,
)
from nanoquant_b200.sharding import RowShardedLinear, row_range, shard_rows, token_range
from oracle import packed_oracle as po


def _oracle_layer(state) -> po.OracleLayer:
    overlay = None
    if isinstance(state, OverlaidLayerState):
        overlay, state = state.overlay, state.base
    assert isinstance(state, PackedLayerState)

    def f(v):
        return None if v is None else v.float().numpy()

    layer = po.OracleLayer(
        state.spec.in_features, state.spec.out_features, state.spec.rank,
        state.left_words.numpy(), state.right_words.numpy(), f(state.scale_pre), f(state.scale_mid),
        f(state.scale_post), f(state.bias),
        None if state.outlier_indices is None else state.outlier_indices.numpy(),
        None if state.outlier_values is None else (
            state.outlier_values.numpy() if state.outlier_values.dtype == torch.int8 else f(state.outlier_values)),
        f(state.outlier_scales), f(state.patch_left), f(state.patch_right),
    )
    if overlay is not None:
        layer.overlay_row_ids = overlay.row_ids.numpy()
        layer.overlay_values = overlay.values.numpy()
        layer.overlay_scales = overlay.scales.float().numpy()
    return layer


class OracleBackend:
    """The per-rank linear of these tests: prepare/linear over the oracle (float64 accumulation)."""

    def prepare(self, state, device):  # noqa: ARG002 - CPU only
        return _oracle_layer(state)

    def linear(self, value: torch.Tensor, layer: po.OracleLayer) -> torch.Tensor:
        out = po.packed_linear(value.float().numpy(), layer, accumulate="float64")
        return torch.from_numpy(np.ascontiguousarray(out, dtype=np.float32))


def _state(n: int, m: int, r: int, seed: int, *, overlay_rows: int = 0):
    """Random layout-v1 layer with 3 int8 salient columns, bias and (optionally) int8 overlay rows."""

    g = torch.Generator().manual_seed(seed)
    spec = QuantizedLinearSpec("blocks.0.r", "nanoquant-v1", n, m, r, "float32", "float16", outlier_count=3,
                               outlier_value_dtype="int8", has_outlier_scales=True, has_bias=True)
    pre = (torch.randn(n, generator=g).abs() * 0.05 + 0.01).half()
    idx = torch.sort(torch.randperm(n, generator=g)[:3]).values
    pre[idx] = 0
    logical = LogicalLayerState(
        spec,
        torch.where(torch.rand(m, r, generator=g) > 0.5, 1.0, -1.0),
        torch.where(torch.rand(r, n, generator=g) > 0.5, 1.0, -1.0),
        pre,
        (torch.randn(r, generator=g).abs() + 0.5).half(),
        (torch.randn(m, generator=g).abs() * 0.05 + 0.01).half(),
        bias=torch.randn(m, generator=g).half(),
        outlier_indices=idx,
        outlier_values=torch.randint(-127, 128, (m, 3), generator=g, dtype=torch.int8),
        outlier_scales=torch.full((3,), 0.002).half(),
    )
    state = pack_logical_layer(logical)
    if overlay_rows:
        g = torch.Generator().manual_seed(seed + 1)
        rows = torch.sort(torch.randperm(m, generator=g)[:overlay_rows]).values.to(torch.int32)
        overlay = OutlierRowOverlay(rows, torch.randint(-127, 128, (overlay_rows, n), generator=g, dtype=torch.int8),
                                    torch.full((overlay_rows,), 0.002, dtype=torch.float16))
        state = OverlaidLayerState(state, overlay)
    return state


def test_token_range_partitions_every_token_once() -> None:
    for total in (0, 1, 7, 32768, 32769):
        for world in (1, 2, 3, 8):
            ranges = [token_range(total, world, g) for g in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            sizes = [hi - lo for lo, hi in ranges]
            assert max(sizes) - min(sizes) <= 1


def test_row_range_uses_whole_tiles() -> None:
    for m in (17, 128, 1000, 4096, 14336):
        for world in (1, 2, 4, 8):
            ranges = [row_range(m, world, g) for g in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == m
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            assert all(lo % 128 == 0 or lo == hi for lo, hi in ranges)  # empty when tiles < ranks


def test_shard_rows_computes_the_same_rows() -> None:
    state = _state(96, 300, 40, seed=3, overlay_rows=9)
    x = torch.randn(5, 96, generator=torch.Generator().manual_seed(1))
    full = OracleBackend().linear(x, _oracle_layer(state))
    for lo, hi in ((0, 128), (128, 256), (256, 300), (0, 300)):
        part = OracleBackend().linear(x, _oracle_layer(shard_rows(state, lo, hi)))
        torch.testing.assert_close(part, full[:, lo:hi], rtol=0, atol=1e-6)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, result_dir: str) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        state = _state(96, 300, 40, seed=3, overlay_rows=9)
        x = torch.randn(6, 96, generator=torch.Generator().manual_seed(4))
        # U row shard + all-gather
        sharded = RowShardedLinear(OracleBackend(), state, "cpu")
        y = sharded(x)
        # token batches: this rank's slice of the tokens, gathered for the check
        lo, hi = token_range(x.shape[0], world, rank)
        local = OracleBackend().linear(x[lo:hi], _oracle_layer(state))
        width = -(-x.shape[0] // world)
        padded = torch.zeros(width, 300)
        padded[: hi - lo] = local
        parts = [torch.empty_like(padded) for _ in range(world)]
        dist.all_gather(parts, padded)
        tokens = torch.cat([p[: b - a] for p, (a, b) in zip(parts, [token_range(x.shape[0], world, g)
                                                                    for g in range(world)])])
        torch.save({"rows": y, "tokens": tokens}, os.path.join(result_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_row_shard_and_token_batches_over_two_gloo_ranks(tmp_path) -> None:
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    state = _state(96, 300, 40, seed=3, overlay_rows=9)
    x = torch.randn(6, 96, generator=torch.Generator().manual_seed(4))
    full = OracleBackend().linear(x, _oracle_layer(state))
    for rank in range(world):
        out = torch.load(tmp_path / f"rank{rank}.pt")
        torch.testing.assert_close(out["rows"], full, rtol=0, atol=1e-6)
        torch.testing.assert_close(out["tokens"], full, rtol=0, atol=1e-6)


def _absent_rank_worker(rank: int, world: int, port: int, result_dir: str) -> None:
    """Rank 1 never joins the row-shard all-gather; rank 0's call must end with an error, not hang."""

    import time
    from datetime import timedelta

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    outcome = "absent"
    try:
        state = _state(96, 300, 40, seed=3)
        sharded = RowShardedLinear(OracleBackend(), state, "cpu")
        if rank == 0:
            start = time.monotonic()
            try:
                sharded(torch.randn(2, 96, generator=torch.Generator().manual_seed(5)))
                outcome = "returned"
            except RuntimeError as error:
                outcome = f"raised after {time.monotonic() - start:.1f}s: {type(error).__name__}"
        else:
            time.sleep(8.0)  # stays alive but never calls the collective
    finally:
        (Path(result_dir) / f"rank{rank}.txt").write_text(outcome)
        dist.destroy_process_group()


@pytest.mark.timeout(180)
def test_row_shard_gather_times_out_when_a_rank_never_joins(tmp_path) -> None:
    world = 2
    mp.spawn(_absent_rank_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    outcome = (tmp_path / "rank0.txt").read_text()
    assert outcome.startswith("raised after"), outcome
    assert float(outcome.split()[2].rstrip("s:")) < 30.0
    assert (tmp_path / "rank1.txt").read_text() == "absent"


if __name__ == "__main__":  # pragma: no cover
    pytest.main([__file__, "-q"])
