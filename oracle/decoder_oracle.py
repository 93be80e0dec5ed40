"""CPU restatement of a Qwen3-style decode step (test infrastructure only).

The checker for ``nanoquant_b200.decoder``: numpy float32 arithmetic (float64
where noted), the packed projections through ``packed_oracle.packed_linear``,
and bf16 rounding (round to nearest even) at the points where the device path
stores bf16: the normalised activations, the rotated queries and keys, the
cache rows and the attention output.  The SwiGLU product stays float32: the
device forms it as the down projection loads its input.  The layer math
follows the reference model shell (``src/nanoquant/runtime/torch_model.py:
185-421``: RMSNorm, per-head q/k RMSNorm, rotate-half RoPE, grouped-query
attention, SwiGLU MLP, residual adds, final norm and lm head).  Only tests
import it.
"""

from __future__ import annotations

import numpy as np

from oracle import packed_oracle as po


def bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to bfloat16 (nearest even), returned as float32."""

    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    # round half to even on the 16 dropped bits (uint32 arithmetic: no finite
    # value carries past bit 31)
    r = (u >> 16) & np.uint32(1)
    r += np.uint32(0x7FFF)
    r += u
    r &= np.uint32(0xFFFF0000)
    return r.view(np.float32)


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    r = 1.0 / np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True) + eps)
    return (x * r.astype(np.float32) * w).astype(np.float32)


def rope_tables(positions: np.ndarray, head_dim: int, theta: float) -> tuple[np.ndarray, np.ndarray]:
    inv = 1.0 / (theta ** (np.arange(0, head_dim, 2, dtype=np.float64) / head_dim))
    angles = positions.astype(np.float64)[:, None] * inv[None, :]
    emb = np.concatenate((angles, angles), axis=-1)
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)


def rotate(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Rotate-half RoPE of ``x [..., head_dim]`` with rows of ``cos``/``sin`` broadcast over heads."""

    half = x.shape[-1] // 2
    rotated = np.concatenate((-x[..., half:], x[..., :half]), axis=-1)
    return (x * cos + rotated * sin).astype(np.float32)


def attention(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, keys: int, window: int = 0) -> np.ndarray:
    """``q [T, Hq, hd]``; caches ``[Hkv, L, hd]``; token t sees rows ``[0, keys + t)`` (float64 math).

    ``window > 0``: only the last ``window`` of those rows (Gemma-3's sliding
    layers mask keys at positions <= query position - window).
    """

    tokens, q_heads, hd = q.shape
    group = q_heads // k_cache.shape[0]
    out = np.zeros((tokens, q_heads, hd), np.float32)
    for t in range(tokens):
        first = max(0, keys + t - window) if window > 0 else 0
        for h in range(q_heads):
            kv = h // group
            k = k_cache[kv, first: keys + t].astype(np.float64)
            v = v_cache[kv, first: keys + t].astype(np.float64)
            s = (k @ q[t, h].astype(np.float64)) / np.sqrt(hd)
            p = np.exp(s - s.max())
            out[t, h] = (p @ v) / p.sum()
    return out


def decode_layer(h: np.ndarray, proj: dict, norms: dict, k_cache: np.ndarray, v_cache: np.ndarray, *,
                 position: int, q_heads: int, kv_heads: int, head_dim: int, eps: float, cos: np.ndarray,
                 sin: np.ndarray, accumulate: str = "float64", xn_bf16: bool = True,
                 sequences: bool = False) -> np.ndarray:
    """One Qwen3-style layer on the residual stream ``h [T, hidden]``; returns the new ``h``.

    ``proj``: ``OracleLayer`` per projection name; ``norms``: this layer's
    ``input_norm``, ``post_norm``, ``q_norm`` and ``k_norm``.  The caches are
    updated in place at rows ``position + t``.  ``xn_bf16``: the normalised
    activations are rounded to bf16 before the projections (the device's
    shell engine stores them as bf16; its fused engine keeps them fp32).
    ``sequences``: token t is the next token of its own sequence, caches
    ``[T, Hkv, L, hd]``, updated at row ``position`` of cache t; each token
    attends to rows ``[0, position]`` of its own caches.
    """

    tokens = h.shape[0]
    rnd = bf16 if xn_bf16 else (lambda value: value)

    def linear(x: np.ndarray, layer) -> np.ndarray:
        return po.packed_linear(x, layer, accumulate=accumulate).astype(np.float32)

    xn = rnd(rmsnorm(h, norms["input_norm"], eps))
    q = linear(xn, proj["q_proj"]).reshape(tokens, q_heads, head_dim)
    k = linear(xn, proj["k_proj"]).reshape(tokens, kv_heads, head_dim)
    v = linear(xn, proj["v_proj"]).reshape(tokens, kv_heads, head_dim)
    q = bf16(rotate(rmsnorm(q, norms["q_norm"], eps), cos[:, None, :], sin[:, None, :]))
    k = bf16(rotate(rmsnorm(k, norms["k_norm"], eps), cos[:, None, :], sin[:, None, :]))
    if sequences:
        for t in range(tokens):
            k_cache[t, :, position] = k[t]
            v_cache[t, :, position] = bf16(v[t])
        a = np.concatenate([attention(q[t:t + 1], k_cache[t], v_cache[t], position + 1) for t in range(tokens)])
        a = bf16(a.reshape(tokens, q_heads * head_dim))
    else:
        for t in range(tokens):
            k_cache[:, position + t] = k[t]
            v_cache[:, position + t] = bf16(v[t])
        a = bf16(attention(q, k_cache, v_cache, position + 1).reshape(tokens, q_heads * head_dim))
    h = h + linear(a, proj["o_proj"])
    xn = rnd(rmsnorm(h, norms["post_norm"], eps))
    gate = linear(xn, proj["gate_proj"])
    up = linear(xn, proj["up_proj"])
    with np.errstate(over="ignore"):  # exp(-gate) overflows to inf for very negative gates: silu -> 0
        act = (gate / (1.0 + np.exp(-gate)) * up).astype(np.float32)
    return h + linear(act, proj["down_proj"])


def decode_step_streaming(hidden: np.ndarray, layer_count: int, layer_at, final_norm: np.ndarray,
                          lm_head: np.ndarray, *, position: int, q_heads: int, kv_heads: int, head_dim: int,
                          eps: float, theta: float, accumulate: str = "float64",
                          head_accumulate: str = "float64", xn_bf16: bool = True,
                          sequences: bool = False) -> np.ndarray:
    """Logits ``[T, vocab]`` of a step whose layers arrive one at a time.

    ``layer_at(i)`` returns ``(proj, norms, k_cache, v_cache)`` of layer i (the
    caches are updated in place), so a caller can build each layer's dense
    signs just before it runs and drop them after: host memory stays at one
    layer for any depth.
    """

    tokens = hidden.shape[0]
    h = hidden.astype(np.float32).copy()
    positions = np.full(tokens, position) if sequences else np.arange(position, position + tokens)
    cos, sin = rope_tables(positions, head_dim, theta)
    for i in range(layer_count):
        proj, norms, k_cache, v_cache = layer_at(i)
        h = decode_layer(h, proj, norms, k_cache, v_cache, position=position, q_heads=q_heads, kv_heads=kv_heads,
                         head_dim=head_dim, eps=eps, cos=cos, sin=sin, accumulate=accumulate, xn_bf16=xn_bf16,
                         sequences=sequences)
    xn = bf16(rmsnorm(h, final_norm, eps))
    if head_accumulate == "float64":
        return (xn.astype(np.float64) @ lm_head.astype(np.float64).T).astype(np.float32)
    return (xn @ np.asarray(lm_head, dtype=np.float32).T).astype(np.float32)


def decode_step(hidden: np.ndarray, layers: list[dict], norms: dict, k_caches: list[np.ndarray],
                v_caches: list[np.ndarray], *, position: int, q_heads: int, kv_heads: int, head_dim: int,
                eps: float, theta: float, xn_bf16: bool = True,
                sequences: bool = False) -> tuple[np.ndarray, list[np.ndarray], list[np.ndarray]]:
    """Logits ``[T, vocab]`` and the updated caches.

    ``layers[i]``: ``OracleLayer`` per projection name; ``norms``: lists
    ``input_norm``, ``post_norm``, ``q_norm``, ``k_norm`` (per layer) and
    ``final_norm``, ``lm_head`` (float32 arrays holding bf16 values).
    ``sequences``: independent sequences with caches ``[T, Hkv, L, hd]``
    (see :func:`decode_layer`).
    """

    k_caches = [c.copy() for c in k_caches]
    v_caches = [c.copy() for c in v_caches]

    def layer_at(i: int):
        per_layer = {name: norms[name][i] for name in ("input_norm", "post_norm", "q_norm", "k_norm")}
        return layers[i], per_layer, k_caches[i], v_caches[i]

    logits = decode_step_streaming(hidden, len(layers), layer_at, norms["final_norm"], norms["lm_head"],
                                   position=position, q_heads=q_heads, kv_heads=kv_heads, head_dim=head_dim, eps=eps,
                                   theta=theta, xn_bf16=xn_bf16, sequences=sequences)
    return logits, k_caches, v_caches


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    """The tanh form of GELU (``gelu_pytorch_tanh``, Gemma-3's MLP activation), in float64."""

    x = x.astype(np.float64)
    return (0.5 * x * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (x + 0.044715 * x ** 3)))).astype(np.float32)


def gemma_decode_layer(h: np.ndarray, proj: dict, norms: dict, k_cache: np.ndarray, v_cache: np.ndarray, *,
                       position: int, q_heads: int, kv_heads: int, head_dim: int, eps: float, cos: np.ndarray,
                       sin: np.ndarray, window: int, accumulate: str = "float64") -> np.ndarray:
    """One Gemma-3 layer on ``h [T, hidden]`` (reference ``runtime/torch_model.py:233-681``, HF Gemma-3 math).

    ``norms`` hold the *effective* weights ``1 + w`` of ``input_norm``,
    ``post_attention_norm``, ``pre_feedforward_norm``, ``post_feedforward_norm``,
    ``q_norm`` and ``k_norm``.  Activations into the projections stay fp32
    (the reference's fp32 decode path); q, k, v and the attention output are
    rounded to bf16 where the device stores them.
    """

    tokens = h.shape[0]

    def linear(x: np.ndarray, layer) -> np.ndarray:
        return po.packed_linear(x, layer, accumulate=accumulate).astype(np.float32)

    xn = rmsnorm(h, norms["input_norm"], eps)
    q = linear(xn, proj["q_proj"]).reshape(tokens, q_heads, head_dim)
    k = linear(xn, proj["k_proj"]).reshape(tokens, kv_heads, head_dim)
    v = linear(xn, proj["v_proj"]).reshape(tokens, kv_heads, head_dim)
    q = bf16(rotate(rmsnorm(q, norms["q_norm"], eps), cos[:, None, :], sin[:, None, :]))
    k = bf16(rotate(rmsnorm(k, norms["k_norm"], eps), cos[:, None, :], sin[:, None, :]))
    for t in range(tokens):
        k_cache[:, position + t] = k[t]
        v_cache[:, position + t] = bf16(v[t])
    a = bf16(attention(q, k_cache, v_cache, position + 1, window).reshape(tokens, q_heads * head_dim))
    h = h + rmsnorm(linear(a, proj["o_proj"]), norms["post_attention_norm"], eps)
    xn = rmsnorm(h, norms["pre_feedforward_norm"], eps)
    act = gelu_tanh(linear(xn, proj["gate_proj"])) * linear(xn, proj["up_proj"])
    return h + rmsnorm(linear(act, proj["down_proj"]), norms["post_feedforward_norm"], eps)


def gemma_decode_step_streaming(hidden: np.ndarray, layer_count: int, layer_at, final_norm: np.ndarray, *,
                                position: int, q_heads: int, kv_heads: int, head_dim: int, eps: float,
                                sliding_window: int = 512, global_every: int = 6, local_theta: float = 1e4,
                                global_theta: float = 1e6, accumulate: str = "float64") -> np.ndarray:
    """Final-normed hidden states ``[T, hidden]`` of a Gemma-3 step from the embedded ``hidden``.

    ``layer_at(i)`` returns ``(proj, norms, k_cache, v_cache)`` of layer i
    (effective ``1 + w`` norm weights; caches updated in place).  Layer i is
    global (full attention, ``global_theta``) when ``(i + 1) % global_every ==
    0``, else local (``sliding_window`` keys, ``local_theta``).
    """

    tokens = hidden.shape[0]
    h = hidden.astype(np.float32).copy()
    positions = np.arange(position, position + tokens)
    tables = {theta: rope_tables(positions, head_dim, theta) for theta in (local_theta, global_theta)}
    for i in range(layer_count):
        is_global = (i + 1) % global_every == 0
        cos, sin = tables[global_theta if is_global else local_theta]
        proj, norms, k_cache, v_cache = layer_at(i)
        h = gemma_decode_layer(h, proj, norms, k_cache, v_cache, position=position, q_heads=q_heads,
                               kv_heads=kv_heads, head_dim=head_dim, eps=eps, cos=cos, sin=sin,
                               window=0 if is_global else sliding_window, accumulate=accumulate)
    return rmsnorm(h, final_norm, eps)


class CpuDecodeStep:
    """A full decode step of a Qwen3- or Gemma-3-shaped decoder on the host cores: the timed CPU baseline.

    The reference's CPU path for one step: its model shell's math (the
    functions above) around ``PackedReferenceBackend.linear`` on every
    projection (``packed_oracle.packed_linear``, fp32 like the reference on
    fp32 inputs), then the dense lm head.  Every step runs all ``layers``
    layers; their packed weights cycle through a pool of ``pool`` distinct
    random layers (dense fp32 signs, unpacked once, as the reference's
    ``prepare`` does), so host memory stays bounded while each layer still
    streams its own ~0.8 GB of dense weights from DRAM.
    """

    def __init__(self, *, layers: int, hidden: int, intermediate: int, q_heads: int, kv_heads: int, head_dim: int,
                 vocab: int, position: int, tokens: int = 1, pool: int = 2, bpw: float = 1.0, seed: int = 0,
                 eps: float = 1e-6, theta: float = 1e6, family: str = "qwen3", sequences: bool = False) -> None:
        rng = np.random.default_rng(seed)
        self.family = family
        self.sequences = sequences
        self.layers, self.tokens, self.position = layers, tokens, position
        self.q_heads, self.kv_heads, self.head_dim, self.eps = q_heads, kv_heads, head_dim, eps
        q, kv = q_heads * head_dim, kv_heads * head_dim
        shapes = {"q_proj": (hidden, q), "k_proj": (hidden, kv), "v_proj": (hidden, kv), "o_proj": (q, hidden),
                  "gate_proj": (hidden, intermediate), "up_proj": (hidden, intermediate),
                  "down_proj": (intermediate, hidden)}

        def words(rows: int, cols: int) -> np.ndarray:
            raw = rng.integers(0, 2**32, size=(rows, po.word_count(cols)), dtype=np.uint64).astype(np.uint32)
            if cols % 32:
                raw[:, -1] &= np.uint32((1 << (cols % 32)) - 1)
            return raw.view(np.int32)

        def scales(size: int) -> np.ndarray:
            return (np.abs(rng.standard_normal(size)) * 0.05 + 0.01).astype(np.float16).astype(np.float32)

        def norm(size: int) -> np.ndarray:
            return bf16((1.0 + 0.02 * rng.standard_normal(size)).astype(np.float32))

        self.pool = []
        for _ in range(pool):
            proj = {}
            for name, (n, m) in shapes.items():
                r = int(bpw * m * n // (m + n))
                layer = po.OracleLayer(n, m, r, words(m, r), words(r, n), scales(n), np.ones(r, np.float32),
                                       scales(m))
                layer.prepared()
                proj[name] = layer
            if family == "gemma":  # effective weights 1 + w of Gemma's norms
                norms = {name: 1.0 + norm(hidden) for name in ("input_norm", "post_attention_norm",
                                                                "pre_feedforward_norm", "post_feedforward_norm")}
                norms.update(q_norm=1.0 + norm(head_dim), k_norm=1.0 + norm(head_dim))
            else:
                norms = {"input_norm": norm(hidden), "post_norm": norm(hidden), "q_norm": norm(head_dim),
                         "k_norm": norm(head_dim)}
            cache = (tokens, kv_heads, position + 1, head_dim) if sequences else (kv_heads, position + tokens, head_dim)
            k = bf16(rng.standard_normal(cache, dtype=np.float32))
            v = bf16(rng.standard_normal(cache, dtype=np.float32))
            self.pool.append((proj, norms, k, v))
        self.final_norm = norm(hidden) + (1.0 if family == "gemma" else 0.0)
        self.theta = theta
        self.hidden = rng.standard_normal((tokens, hidden), dtype=np.float32)
        if family == "gemma":  # no vocabulary head
            self.lm_head = None
            return
        # the 0.6 G-entry head: torch's generator and bf16 rounding (round to
        # nearest even, as bf16() above) are several times faster than numpy's here
        import torch

        head = torch.randn(vocab, hidden, generator=torch.Generator().manual_seed(seed + 1)) * 0.02
        self.lm_head = head.bfloat16().float().numpy()

    def step(self) -> np.ndarray:
        if self.family == "gemma":
            pool = self.pool
            return gemma_decode_step_streaming(self.hidden, self.layers, lambda i: pool[i % len(pool)],
                                               self.final_norm, position=self.position, q_heads=self.q_heads,
                                               kv_heads=self.kv_heads, head_dim=self.head_dim, eps=self.eps,
                                               accumulate="float32")
        pool = self.pool
        return decode_step_streaming(self.hidden, self.layers, lambda i: pool[i % len(pool)], self.final_norm,
                                     self.lm_head, position=self.position, q_heads=self.q_heads,
                                     kv_heads=self.kv_heads, head_dim=self.head_dim, eps=self.eps, theta=self.theta,
                                     accumulate="float32", head_accumulate="float32", sequences=self.sequences)


__all__ = ["CpuDecodeStep", "attention", "bf16", "decode_layer", "decode_step", "decode_step_streaming",
           "gelu_tanh", "gemma_decode_layer", "gemma_decode_step_streaming", "rmsnorm", "rope_tables", "rotate"]
