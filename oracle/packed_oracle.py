"""CPU oracle for NanoQuant's packed binary low-rank linear.

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped package imports this module:
only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may use it, and only as the checker
or the timed CPU baseline, never as the thing measured for the GPU path.

It restates, in numpy, the reference's own CPU path for this operator:

* layout-v1 sign packing -- ``src/nanoquant/runtime/packed.py:139-218``;
* the packed reference backend -- ``PackedReferenceBackend.prepare/linear``,
  ``src/nanoquant/runtime/reference.py:184-235``, with the salient masking of
  ``reference.py:101-106`` and the int8 salient scaling of ``reference.py:93-98``;
* the product-codebook decode -- ``src/nanoquant/runtime/product_codebook.py:110-143``;
* the mixed-V record stream -- ``src/nanoquant/runtime/mixed_v.py:75-165``.

Pinning: ``tests/golden/*.npz`` hold inputs and outputs produced by running the
reference itself (``tests/golden/make_golden.py`` imports it from the reference
tree); ``tests/test_oracle.py`` checks this module against every fixture.  The
int8 residual-row overlay has no reference type, so :func:`apply_row_overlay`
is unpinned (it restates the cost model's definition in
``src/nanoquant/domain/structured_sidecar.py:32-118``).

Arithmetic follows the reference: the reference computes in the input dtype, so
fp32 inputs give fp32 matmuls (numpy/BLAS sgemm here, torch sgemm there).
``accumulate="float64"`` is offered for size-independent error analysis.
"""

from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field

import numpy as np

WORD_BITS = 32

# byte value -> its 8 columns as +/-1 (bit j of the byte is column j; 1 = -1)
_BYTE_SIGNS = (1.0 - 2.0 * ((np.arange(256)[:, None] >> np.arange(8)) & 1)).astype(np.float32)
_THREADS = max(1, min(32, os.cpu_count() or 1))
_POOL: ThreadPoolExecutor | None = None


def _pool() -> ThreadPoolExecutor:
    global _POOL
    if _POOL is None:
        _POOL = ThreadPoolExecutor(_THREADS)
    return _POOL


# ---------------------------------------------------------------- layout v1 ---

def word_count(columns: int) -> int:
    """``packed_word_count`` (reference packed.py:139-142)."""

    if columns <= 0:
        raise ValueError("packed sign column count must be positive")
    return (columns + WORD_BITS - 1) // WORD_BITS


def pack_signs(signs: np.ndarray) -> np.ndarray:
    """``pack_sign_matrix`` (reference packed.py:170-188): bit c%32 of word c//32, 1 = -1.

    Written as an explicit shift-and-sum over the 32 lanes of each word.
    """

    signs = np.asarray(signs)
    if signs.ndim != 2 or signs.shape[0] == 0 or signs.shape[1] == 0:
        raise ValueError("logical sign matrix dimensions must be positive")
    if not np.all((signs == 1) | (signs == -1)):
        raise ValueError("logical signs contain a value other than -1 or +1")
    rows, columns = signs.shape
    words = word_count(columns)
    negative = np.zeros((rows, words * WORD_BITS), dtype=np.uint64)
    negative[:, :columns] = signs < 0
    lanes = np.arange(WORD_BITS, dtype=np.uint64)
    packed = (negative.reshape(rows, words, WORD_BITS) << lanes).sum(axis=-1, dtype=np.uint64)
    return packed.astype(np.uint32).view(np.int32)


def padding_is_zero(words: np.ndarray, columns: int) -> bool:
    """Tail-bit check of ``_validate_packed_matrix`` (reference packed.py:191-201)."""

    tail = columns % WORD_BITS
    if tail == 0:
        return True
    last = np.asarray(words)[:, -1].view(np.uint32).astype(np.uint64)
    return not bool(np.any(last & np.uint64(0xFFFFFFFF ^ ((1 << tail) - 1))))


def unpack_signs(words: np.ndarray, rows: int, columns: int) -> np.ndarray:
    """``unpack_sign_matrix`` (reference packed.py:204-218) as fp32 +/-1."""

    words = np.asarray(words)
    if words.dtype != np.int32 or words.shape != (rows, word_count(columns)):
        raise ValueError("packed sign matrix must be int32 [rows, ceil(columns/32)]")
    if not padding_is_zero(words, columns):
        raise ValueError("packed sign matrix has a non-zero padding bit")
    # little-endian words: byte b of word w holds columns 32w + 8b .. 32w + 8b + 7,
    # least significant bit first, so each byte expands to its 8 columns in
    # order through a 256-entry table of +/-1 rows (threads take row blocks:
    # the copy is bound by first touches of the output pages)
    raw = np.ascontiguousarray(words).view(np.uint8)
    out = np.empty((rows, raw.shape[1] * 8), dtype=np.float32)
    block = max(1, -(-rows // (4 * _THREADS)))

    def expand(lo: int) -> None:
        hi = min(rows, lo + block)
        np.take(_BYTE_SIGNS, raw[lo:hi], axis=0, out=out[lo:hi].reshape(hi - lo, -1, 8))

    if rows * raw.shape[1] < (1 << 16):
        for lo in range(0, rows, block):
            expand(lo)
    else:
        list(_pool().map(expand, range(0, rows, block)))
    return out if out.shape[1] == columns else np.ascontiguousarray(out[:, :columns])


# ----------------------------------------------------------- packed layer ---

@dataclass
class OracleLayer:
    """Plain-array description of one packed layer (the fields of ``PackedLayerState``)."""

    in_features: int
    out_features: int
    rank: int
    left_words: np.ndarray   # U [out, ceil(rank/32)] int32
    right_words: np.ndarray  # V [rank, ceil(in/32)] int32
    scale_pre: np.ndarray
    scale_mid: np.ndarray
    scale_post: np.ndarray
    bias: np.ndarray | None = None
    outlier_indices: np.ndarray | None = None
    outlier_values: np.ndarray | None = None
    outlier_scales: np.ndarray | None = None
    patch_left: np.ndarray | None = None
    patch_right: np.ndarray | None = None
    # row overlay (no reference type)
    overlay_row_ids: np.ndarray | None = None
    overlay_values: np.ndarray | None = None
    overlay_scales: np.ndarray | None = None
    _dense: dict = field(default_factory=dict, repr=False)

    def prepared(self) -> dict:
        """``PackedReferenceBackend.prepare``: unpack once to dense +/-1 (reference reference.py:199-206)."""

        if not self._dense:
            self._dense["left"] = unpack_signs(self.left_words, self.out_features, self.rank)
            self._dense["right"] = unpack_signs(self.right_words, self.rank, self.in_features)
        return self._dense


def _f(value: np.ndarray | None, dtype) -> np.ndarray | None:
    return None if value is None else np.asarray(value).astype(dtype, copy=False)


def masked_scale_pre(layer: OracleLayer) -> np.ndarray:
    """``_masked_scale_pre`` (reference reference.py:101-106): zero pre at salient columns."""

    pre = np.array(layer.scale_pre, dtype=np.float32)
    if layer.outlier_indices is not None and len(layer.outlier_indices):
        pre[np.asarray(layer.outlier_indices, dtype=np.int64)] = 0
    return pre


def outlier_weights(layer: OracleLayer) -> np.ndarray | None:
    """``_outlier_values`` (reference reference.py:93-98): int8 values times per-column scales."""

    if layer.outlier_values is None:
        return None
    if layer.outlier_scales is None:
        return np.asarray(layer.outlier_values).astype(np.float32)
    return np.asarray(layer.outlier_values).astype(np.float32) * np.asarray(layer.outlier_scales).astype(np.float32)


def packed_linear(x: np.ndarray, layer: OracleLayer, *, accumulate: str = "float32") -> np.ndarray:
    """``PackedReferenceBackend.linear`` (reference reference.py:208-235) on fp32 input.

    ``x`` is ``[..., in]``; returns ``[..., out]`` in the accumulate dtype.
    Operation order follows the reference: latent, stage 2, salient term,
    low-rank patch, bias; the row overlay (not in the reference) is added last.
    """

    dt = np.float64 if accumulate == "float64" else np.float32
    x = np.asarray(x, dtype=np.float32).astype(dt, copy=False)
    lead = x.shape[:-1]
    x2 = x.reshape(-1, layer.in_features)
    dense = layer.prepared()
    # like torch's ``.to(dtype)``, no copy when the dtype already matches
    pre = masked_scale_pre(layer).astype(dt, copy=False)
    right = dense["right"].astype(dt, copy=False)
    left = dense["left"].astype(dt, copy=False)
    latent = (x2 * pre) @ right.T
    output = (latent * _f(layer.scale_mid, dt)) @ (left * _f(layer.scale_post, dt)[:, None]).T
    weights = outlier_weights(layer)
    if layer.outlier_indices is not None and weights is not None:
        columns = np.asarray(layer.outlier_indices, dtype=np.int64)
        output = output + x2[:, columns] @ weights.astype(dt).T
    if layer.patch_left is not None and layer.patch_right is not None:
        output = output + (x2 @ _f(layer.patch_right, dt).T) @ _f(layer.patch_left, dt).T
    if layer.bias is not None:
        output = output + _f(layer.bias, dt)
    output = apply_row_overlay(x2, output, layer, dt)
    return output.reshape(*lead, layer.out_features)


def apply_row_overlay(x2: np.ndarray, output: np.ndarray, layer: OracleLayer, dt=np.float32) -> np.ndarray:
    """Int8 residual rows: ``y[:, ids[j]] += scale[j] * (x @ R[j])``.  Parity unpinned (no reference type)."""

    if layer.overlay_row_ids is None:
        return output
    ids = np.asarray(layer.overlay_row_ids, dtype=np.int64)
    residual = (x2 @ np.asarray(layer.overlay_values).astype(dt).T) * _f(layer.overlay_scales, dt)
    output = np.array(output, copy=True)
    output[:, ids] += residual
    return output


# -------------------------------------------------------- product codebook ---

def unpack_codebook_records(payload: np.ndarray, count: int) -> np.ndarray:
    """16-bit record stream, two per word, low half first (reference product_codebook.py:59-81)."""

    unsigned = np.asarray(payload).view(np.uint32).astype(np.uint64)
    low = unsigned & np.uint64(0xFFFF)
    high = unsigned >> np.uint64(16)
    records = np.stack((low, high), axis=1).reshape(-1)
    if count % 2 and records[count] != 0:
        raise ValueError("product-codebook payload has a non-zero padding record")
    return records[:count].astype(np.uint32)


def decode_codebook_right_words(
    free_words: np.ndarray,
    payload: np.ndarray,
    first: np.ndarray,
    second: np.ndarray,
    rank: int,
    columns: int,
) -> np.ndarray:
    """``decode_product_codebook_right_words`` (reference product_codebook.py:110-143)."""

    free_words = np.asarray(free_words)
    free_rows = free_words.shape[0]
    per_row = word_count(columns)
    records = unpack_codebook_records(payload, (rank - free_rows) * per_row)
    table_lo = np.asarray(first).view(np.uint16).astype(np.uint32)
    table_hi = np.asarray(second).view(np.uint16).astype(np.uint32)
    coded = table_lo[records & 0xFF] | (table_hi[records >> 8] << 16)
    coded = coded.astype(np.uint32).view(np.int32).reshape(rank - free_rows, per_row)
    words = np.concatenate((free_words, coded), axis=0)
    if not padding_is_zero(words, columns):
        raise ValueError("packed sign matrix has a non-zero padding bit")
    return words


# ------------------------------------------------------------- mixed V ---

MIXED_V_RECORD_BITS = 19
MIXED_V_INDEX_BITS = 10


def mixed_v_pair_table() -> np.ndarray:
    """Pair id -> (first | second << 8) over the 496 bit pairs (reference mixed_v.py:34-48)."""

    pairs = [(a, b) for a in range(WORD_BITS) for b in range(a + 1, WORD_BITS)]
    table = np.zeros(1 << 9, dtype=np.int32)
    for pair_id, (a, b) in enumerate(pairs):
        table[pair_id] = a | (b << 8)
    return table


def unpack_mixed_v_records(payload: np.ndarray, count: int) -> tuple[np.ndarray, np.ndarray]:
    """19-bit record stream (reference mixed_v.py:104-140) -> (codebook index, pair id)."""

    unsigned = np.asarray(payload).view(np.uint32).astype(np.uint64)
    offsets = np.arange(count, dtype=np.uint64) * np.uint64(MIXED_V_RECORD_BITS)
    word = (offsets // np.uint64(WORD_BITS)).astype(np.int64)
    shift = offsets % np.uint64(WORD_BITS)
    extended = np.concatenate((unsigned, np.zeros(1, dtype=np.uint64)))
    both = extended[word] | (extended[word + 1] << np.uint64(WORD_BITS))
    records = (both >> shift) & np.uint64((1 << MIXED_V_RECORD_BITS) - 1)
    return (records & np.uint64(1023)).astype(np.int32), (records >> np.uint64(10)).astype(np.int32)


def decode_mixed_v_right_words(free_words, payload, codebook, rank: int, columns: int) -> np.ndarray:
    """``decode_mixed_v_right_words`` (reference mixed_v.py:143-165)."""

    free_words = np.asarray(free_words)
    per_row = word_count(columns)
    count = (rank - free_words.shape[0]) * per_row
    index, pair = unpack_mixed_v_records(payload, count)
    table = mixed_v_pair_table()[pair].astype(np.uint32)
    mask = (np.uint32(1) << (table & 0xFF)) | (np.uint32(1) << ((table >> 8) & 0xFF))
    base = np.asarray(codebook).view(np.uint32)[index]
    coded = (base ^ mask).astype(np.uint32).view(np.int32).reshape(-1, per_row)
    return np.concatenate((free_words, coded), axis=0)
