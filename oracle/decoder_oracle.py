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

    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return r.astype(np.uint32).view(np.float32)


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


def attention(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, keys: int) -> np.ndarray:
    """``q [T, Hq, hd]``; caches ``[Hkv, L, hd]``; token t sees rows ``[0, keys + t)`` (float64 math)."""

    tokens, q_heads, hd = q.shape
    group = q_heads // k_cache.shape[0]
    out = np.zeros((tokens, q_heads, hd), np.float32)
    for t in range(tokens):
        for h in range(q_heads):
            kv = h // group
            k = k_cache[kv, : keys + t].astype(np.float64)
            v = v_cache[kv, : keys + t].astype(np.float64)
            s = (k @ q[t, h].astype(np.float64)) / np.sqrt(hd)
            p = np.exp(s - s.max())
            out[t, h] = (p @ v) / p.sum()
    return out


def decode_step(hidden: np.ndarray, layers: list[dict], norms: dict, k_caches: list[np.ndarray],
                v_caches: list[np.ndarray], *, position: int, q_heads: int, kv_heads: int, head_dim: int,
                eps: float, theta: float) -> tuple[np.ndarray, list[np.ndarray], list[np.ndarray]]:
    """Logits ``[T, vocab]`` and the updated caches.

    ``layers[i]``: ``OracleLayer`` per projection name; ``norms``: lists
    ``input_norm``, ``post_norm``, ``q_norm``, ``k_norm`` (per layer) and
    ``final_norm``, ``lm_head`` (float32 arrays holding bf16 values).
    """

    tokens = hidden.shape[0]
    h = hidden.astype(np.float32).copy()
    cos, sin = rope_tables(np.arange(position, position + tokens), head_dim, theta)
    k_caches = [c.copy() for c in k_caches]
    v_caches = [c.copy() for c in v_caches]

    def linear(x: np.ndarray, layer) -> np.ndarray:
        return po.packed_linear(x, layer, accumulate="float64").astype(np.float32)

    for i, proj in enumerate(layers):
        xn = bf16(rmsnorm(h, norms["input_norm"][i], eps))
        q = linear(xn, proj["q_proj"]).reshape(tokens, q_heads, head_dim)
        k = linear(xn, proj["k_proj"]).reshape(tokens, kv_heads, head_dim)
        v = linear(xn, proj["v_proj"]).reshape(tokens, kv_heads, head_dim)
        q = bf16(rotate(rmsnorm(q, norms["q_norm"][i], eps), cos[:, None, :], sin[:, None, :]))
        k = bf16(rotate(rmsnorm(k, norms["k_norm"][i], eps), cos[:, None, :], sin[:, None, :]))
        for t in range(tokens):
            k_caches[i][:, position + t] = k[t]
            v_caches[i][:, position + t] = bf16(v[t])
        a = bf16(attention(q, k_caches[i], v_caches[i], position + 1).reshape(tokens, q_heads * head_dim))
        h = h + linear(a, proj["o_proj"])
        xn = bf16(rmsnorm(h, norms["post_norm"][i], eps))
        gate = linear(xn, proj["gate_proj"])
        up = linear(xn, proj["up_proj"])
        act = (gate / (1.0 + np.exp(-gate)) * up).astype(np.float32)
        h = h + linear(act, proj["down_proj"])
    xn = bf16(rmsnorm(h, norms["final_norm"], eps))
    logits = (xn.astype(np.float64) @ norms["lm_head"].astype(np.float64).T).astype(np.float32)
    return logits, k_caches, v_caches


__all__ = ["attention", "bf16", "decode_step", "rmsnorm", "rope_tables", "rotate"]
