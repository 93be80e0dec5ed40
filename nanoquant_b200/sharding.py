"""Multi-GPU partitions of the packed linear (prefill).

Two partitions; both are exact — every output element is computed by exactly
one rank with the same arithmetic as the unsharded call:

* **Token batches** (:func:`token_range`): rank g of G takes tokens
  ``[g*T/G, (g+1)*T/G)`` and a full replica of the weights.  Prefill batches
  are independent, so there is no collective on the data path.
* **U row shard** (:class:`RowShardedLinear`): every rank runs stage 1 in full
  (all of V, the whole latent) and stage 2 on its rows ``[r0, r1)`` of U
  (with their ``scale_post``, bias, salient-column weights, low-rank patch rows
  and int8 overlay rows); one all-gather of the fp32 ``y`` slices over NCCL
  joins them.  Row ranges are multiples of the 128-row tensor-core tile.

The reference has no multi-GPU path for this operator; prefill is split by
disjoint token batches, with an optional row shard of U joined by an NCCL
all-gather.
"""

from __future__ import annotations

from dataclasses import replace

import torch

from nanoquant_b200.backend import PreparedLayer
from nanoquant_b200.mixed_v import MixedVLayerState
from nanoquant_b200.overlay import OutlierRowOverlay, OverlaidLayerState
from nanoquant_b200.packed import PackedLayerState
from nanoquant_b200.product_codebook import ProductCodebookLayerState

TILE_ROWS = 128


def token_range(total_tokens: int, world: int, rank: int) -> tuple[int, int]:
    """``[start, stop)`` of rank ``rank``'s token batch; sizes differ by at most one."""

    if world < 1 or not 0 <= rank < world or total_tokens < 0:
        raise ValueError("token_range needs 0 <= rank < world and a non-negative token count")
    base, extra = divmod(total_tokens, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def row_range(out_features: int, world: int, rank: int, multiple: int = TILE_ROWS) -> tuple[int, int]:
    """``[start, stop)`` of rank ``rank``'s output rows: whole ``multiple``-row tiles, last rank takes the tail.

    A rank may get an empty range when there are fewer tiles than ranks.
    """

    if world < 1 or not 0 <= rank < world or out_features <= 0 or multiple <= 0:
        raise ValueError("row_range needs 0 <= rank < world, positive out_features and multiple")
    tiles = -(-out_features // multiple)
    first, last = token_range(tiles, world, rank)
    return min(first * multiple, out_features), min(last * multiple, out_features)


def shard_rows(state: PackedLayerState | OverlaidLayerState | ProductCodebookLayerState | MixedVLayerState,
               start: int, stop: int) -> PackedLayerState | OverlaidLayerState:
    """The layer restricted to output rows ``[start, stop)`` (stage 1 unchanged).

    Product-codebook and mixed-V layers are decoded to layout v1 first (their
    V is the stage-1 factor, kept whole; only U rows are sliced).
    """

    if isinstance(state, OverlaidLayerState):
        base = shard_rows(state.base, start, stop)
        assert isinstance(base, PackedLayerState)
        ids = state.overlay.row_ids.to(torch.int64)
        keep = (ids >= start) & (ids < stop)
        if not bool(keep.any()):
            return base
        overlay = OutlierRowOverlay((ids[keep] - start).to(torch.int32).contiguous(),
                                    state.overlay.values[keep].contiguous(), state.overlay.scales[keep].contiguous())
        return OverlaidLayerState(base, overlay)
    if isinstance(state, (ProductCodebookLayerState, MixedVLayerState)):
        state = state.to_packed()
    if not isinstance(state, PackedLayerState):
        raise TypeError("shard_rows takes packed, mixed-V, product-codebook or overlaid layers")
    spec = state.spec
    if not 0 <= start < stop <= spec.out_features:
        raise ValueError("row shard must be a non-empty range inside the output rows")

    def rows(value: torch.Tensor | None) -> torch.Tensor | None:
        return None if value is None else value[start:stop].contiguous()

    return PackedLayerState(
        replace(spec, out_features=stop - start),
        state.layout,
        rows(state.left_words),
        state.right_words,
        state.scale_pre,
        state.scale_mid,
        rows(state.scale_post),
        bias=rows(state.bias),
        outlier_indices=state.outlier_indices,
        outlier_values=rows(state.outlier_values),
        outlier_scales=state.outlier_scales,
        patch_left=rows(state.patch_left),
        patch_right=state.patch_right,
    )


class RowShardedLinear:
    """One packed linear split over the ranks of ``group`` by U rows.

    ``backend`` prepares this rank's shard on ``device``; calling the object
    runs the local linear and all-gathers the fp32 slices into the full
    ``[..., out_features]`` output (identical on every rank).
    """

    def __init__(self, backend, state, device: torch.device | str, *, group=None, world: int | None = None,
                 rank: int | None = None) -> None:
        import torch.distributed as dist

        self.group = group
        self.world = world if world is not None else dist.get_world_size(group)
        self.rank = rank if rank is not None else dist.get_rank(group)
        self.out_features = state.spec.out_features
        self.ranges = [row_range(self.out_features, self.world, g) for g in range(self.world)]
        self.width = max(stop - start for start, stop in self.ranges)
        start, stop = self.ranges[self.rank]
        self.backend = backend
        self.local: PreparedLayer | None = (backend.prepare(shard_rows(state, start, stop), device)
                                            if stop > start else None)
        self.device = torch.device(device)

    def __call__(self, value: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist

        lead = value.shape[:-1]
        start, stop = self.ranges[self.rank]
        padded = torch.zeros((*lead, self.width), dtype=torch.float32, device=value.device)
        if self.local is not None:
            padded[..., : stop - start] = self.backend.linear(value, self.local)
        parts = [torch.empty_like(padded) for _ in range(self.world)]
        dist.all_gather(parts, padded, group=self.group)
        return torch.cat([part[..., : hi - lo] for part, (lo, hi) in zip(parts, self.ranges)], dim=-1)


__all__ = ["RowShardedLinear", "TILE_ROWS", "row_range", "shard_rows", "token_range"]
