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
               start: int, stop: int, *, pad_to: int | None = None) -> PackedLayerState | OverlaidLayerState:
    """The layer restricted to output rows ``[start, stop)`` (stage 1 unchanged).

    Product-codebook and mixed-V layers are decoded to layout v1 first (their
    V is the stage-1 factor, kept whole; only U rows are sliced).  With
    ``pad_to`` the shard gets ``pad_to - (stop - start)`` extra rows of zero
    words and zero scale, bias, salient and patch weights, which compute
    exactly 0; ``start == stop`` is then allowed (a rank without rows).
    """

    if isinstance(state, OverlaidLayerState):
        base = shard_rows(state.base, start, stop, pad_to=pad_to)
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
    rows_out = stop - start if pad_to is None else pad_to
    if not 0 <= start <= stop <= spec.out_features or rows_out < stop - start or rows_out <= 0:
        raise ValueError("row shard must be a non-empty range inside the output rows")
    extra = rows_out - (stop - start)

    def rows(value: torch.Tensor | None) -> torch.Tensor | None:
        if value is None:
            return None
        part = value[start:stop]
        if extra:
            part = torch.cat((part, torch.zeros((extra, *value.shape[1:]), dtype=value.dtype, device=value.device)))
        return part.contiguous()

    return PackedLayerState(
        replace(spec, out_features=rows_out),
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


class RowShardWork:
    """An all-gather of one :class:`RowShardedLinear` call in flight.

    ``wait()`` orders the caller's current stream after the gather (on CUDA; on
    the CPU the gather has already finished); ``result()`` waits and returns
    the full ``[..., out_features]`` output.
    """

    def __init__(self, owner: "RowShardedLinear", buffer: torch.Tensor, lead: tuple[int, ...], event, work) -> None:
        self.owner, self.buffer, self.lead, self.event, self.work = owner, buffer, lead, event, work

    def wait(self) -> torch.Tensor:
        """Waits for the gather; returns the gathered ``[world, tokens, width]`` buffer (no copy)."""

        if self.event is not None:
            torch.cuda.current_stream(self.buffer.device).wait_event(self.event)
        elif self.work is not None:
            self.work.wait()
        return self.buffer

    def result(self) -> torch.Tensor:
        gathered = self.wait()
        world, tokens, width = gathered.shape
        m = self.owner.out_features
        if tokens == 1:  # decode: the rank slots already sit in output order
            flat = gathered.view(1, world * width)[:, :m]
        else:  # one transposing copy: rank-major slots -> token-major rows
            flat = gathered.permute(1, 0, 2).reshape(tokens, world * width)[:, :m]
        return flat.reshape(*self.lead, m)


class RowShardedLinear:
    """One packed linear split over the ranks of ``group`` by U rows.

    Every rank runs stage 1 in full and stage 2 on its whole 128-row tiles of
    U, padded with zero rows to the widest rank's row count, so each rank's
    slice of the output has one shape.  The local slice is written straight
    into this rank's slot of a preallocated ``[world, tokens, width]`` buffer,
    and one in-place ``all_gather_into_tensor`` fills the other slots; on CUDA
    the gather runs on a side stream, so :meth:`start` returns while it is in
    flight and the caller's next kernels overlap it.  Calling the object runs
    :meth:`start` and returns the full output (identical on every rank).
    """

    def __init__(self, backend, state, device: torch.device | str, *, group=None, world: int | None = None,
                 rank: int | None = None, stream: torch.cuda.Stream | None = None) -> None:
        import torch.distributed as dist

        self.group = group
        self.world = world if world is not None else dist.get_world_size(group)
        self.rank = rank if rank is not None else dist.get_rank(group)
        self.out_features = state.spec.out_features
        self.ranges = [row_range(self.out_features, self.world, g) for g in range(self.world)]
        self.width = max(stop - start for start, stop in self.ranges)
        start, stop = self.ranges[self.rank]
        self.backend = backend
        self.local: PreparedLayer = backend.prepare(shard_rows(state, start, stop, pad_to=self.width), device)
        self.device = torch.device(device)
        self._buffers: dict[int, torch.Tensor] = {}
        # the gather stream (several sharded linears may share one)
        self._stream = (stream or torch.cuda.Stream(self.device)) if self.device.type == "cuda" else None

    def buffer(self, tokens: int) -> torch.Tensor:
        """The gather buffer ``[world, tokens, width]`` for ``tokens`` tokens (kept across calls)."""

        buf = self._buffers.get(tokens)
        if buf is None:
            buf = torch.empty((self.world, tokens, self.width), dtype=torch.float32, device=self.device)
            self._buffers[tokens] = buf
        return buf

    def start(self, value: torch.Tensor) -> RowShardWork:
        """Local rows into this rank's slot, then the all-gather (asynchronous on CUDA)."""

        import torch.distributed as dist

        lead = tuple(value.shape[:-1])
        tokens = value.numel() // value.shape[-1]
        buf = self.buffer(tokens)
        slot = buf[self.rank]
        linear_into = getattr(self.backend, "linear_into", None)
        if linear_into is not None:
            linear_into(value.reshape(tokens, value.shape[-1]), self.local, slot)
        else:
            slot.copy_(self.backend.linear(value, self.local).reshape(tokens, self.width))
        if self._stream is None:
            work = dist.all_gather_into_tensor(buf.view(-1), slot.reshape(-1), group=self.group, async_op=True)
            work.wait()
            return RowShardWork(self, buf, lead, None, None)
        current = torch.cuda.current_stream(self.device)
        self._stream.wait_stream(current)
        with torch.cuda.stream(self._stream):
            dist.all_gather_into_tensor(buf.view(-1), slot.reshape(-1), group=self.group)
            done = torch.cuda.Event()
            done.record(self._stream)
        buf.record_stream(self._stream)
        return RowShardWork(self, buf, lead, done, None)

    def __call__(self, value: torch.Tensor) -> torch.Tensor:
        return self.start(value).result()


__all__ = ["RowShardWork", "RowShardedLinear", "TILE_ROWS", "row_range", "shard_rows", "token_range"]
