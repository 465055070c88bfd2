"""Shared numpy building blocks of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Every function is an f32 restatement of a candle op or a reference helper on
the encoder forward path; the reference call site is cited on each.
"""
from __future__ import annotations

import math

import numpy as np

# crates/inl-core/src/attention.rs:29 — finite additive mask value.
MASK_VALUE = np.float32(-1e4)


def rms_norm(x: np.ndarray, weight: np.ndarray | None, eps: float) -> np.ndarray:
    """``x / sqrt(mean(x^2) + eps) * weight`` over the last axis.

    Restates candle_nn::ops::rms_norm as the reference calls it
    (crates/inl-text/src/qwen3/mod.rs:86-90) and as its textbook test pins it
    (crates/inl-text/src/qwen3/mod.rs:705-730).
    """
    x = x.astype(np.float32, copy=False)
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    y = x / np.sqrt(var + np.float32(eps))
    if weight is not None:
        y = y * weight.astype(np.float32, copy=False)
    return y.astype(np.float32, copy=False)


def layer_norm(x: np.ndarray, weight: np.ndarray, bias: np.ndarray | None, eps: float) -> np.ndarray:
    """``(x - mean) / sqrt(var + eps) * w (+ b)``, biased variance.

    Restates the reference LayerNorm (crates/inl-sparse/src/modernbert.rs:176-209,
    textbook test :1551-1584).
    """
    x = x.astype(np.float32, copy=False)
    mu = np.mean(x, axis=-1, keepdims=True, dtype=np.float32)
    xc = x - mu
    var = np.mean(xc * xc, axis=-1, keepdims=True, dtype=np.float32)
    y = xc / np.sqrt(var + np.float32(eps)) * weight
    if bias is not None:
        y = y + bias
    return y.astype(np.float32, copy=False)


def rope_table(head_dim: int, theta: float, positions: int) -> tuple[np.ndarray, np.ndarray]:
    """cos/sin ``[positions, head_dim/2]`` computed in f64 then stored f32.

    Restates RotaryTable::new (crates/inl-text/src/qwen3/mod.rs:129-153):
    ``inv_freq_i = 1 / theta^(2i/d)``, angle = position * inv_freq.
    """
    half = head_dim // 2
    inv = np.array([1.0 / theta ** ((2 * i) / head_dim) for i in range(half)], dtype=np.float64)
    ang = np.arange(positions, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Half-split rotation ``x*[cos,cos] + rotate_half(x)*[sin,sin]``.

    ``x``: [..., L, heads, d]; ``cos``/``sin``: [L, d/2]. Restates the manual
    rotation the reference pins the fused kernel against
    (crates/inl-text/src/qwen3/mod.rs:160-178, test :677-703).
    """
    half = x.shape[-1] // 2
    x1 = x[..., :half]
    x2 = x[..., half:]
    c = cos[:, None, :]
    s = sin[:, None, :]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1).astype(np.float32)


def silu(x: np.ndarray) -> np.ndarray:
    """candle Activation::Silu (crates/inl-text/src/qwen3/mod.rs:112)."""
    return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def gelu_erf(x: np.ndarray) -> np.ndarray:
    """Exact GELU ``0.5 x (1 + erf(x/sqrt 2))`` (crates/inl-sparse/src/modernbert.rs:426)."""
    from scipy.special import erf  # scipy is test-only tooling here

    return (0.5 * x * (1.0 + erf(x / math.sqrt(2.0)))).astype(np.float32)


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    """tanh-approximated GELU (crates/inl-text/src/gemma2.rs:251)."""
    c = np.float32(math.sqrt(2.0 / math.pi))
    return (0.5 * x * (1.0 + np.tanh(c * (x + np.float32(0.044715) * x * x * x)))).astype(np.float32)


def softmax(x: np.ndarray, axis: int = -1) -> np.ndarray:
    """candle softmax_last_dim: max-subtracted exp over the last axis."""
    m = np.max(x, axis=axis, keepdims=True)
    e = np.exp(x - m)
    return (e / np.sum(e, axis=axis, keepdims=True)).astype(np.float32)


def attend_text(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float,
                causal: bool, window: int | None = None,
                mask_value: np.float32 = MASK_VALUE) -> np.ndarray:
    """Attention for ONE text, no padding: ``softmax(scale*q k^T + mask) v``.

    q: [L, Hq, d]; k, v: [L, Hkv, d] (GQA: query head h reads kv head
    h // (Hq/Hkv), restating repeat_kv, crates/inl-core/src/attention.rs:202-210).
    ``causal`` adds ``mask_value`` for key > query
    (crates/inl-core/src/attention.rs:170-199); ``window`` adds it where
    |query - key| > window (ModernBERT local layers,
    crates/inl-sparse/src/modernbert.rs:543,607; Gemma sliding layers,
    crates/inl-text/src/gemma2.rs:499-523). Packing removes the padding mask.
    Returns [L, Hq, d].
    """
    L, hq, d = q.shape
    hkv = k.shape[1]
    rep = hq // hkv
    kk = np.repeat(k, rep, axis=1)
    vv = np.repeat(v, rep, axis=1)
    s = np.einsum("qhd,khd->hqk", q, kk, dtype=np.float32) * np.float32(scale)
    if causal or window is not None:
        qi = np.arange(L)[:, None]
        ki = np.arange(L)[None, :]
        add = np.zeros((L, L), dtype=np.float32)
        if causal:
            add += np.where(ki > qi, mask_value, np.float32(0))
        if window is not None:
            add += np.where(np.abs(qi - ki) > window, mask_value, np.float32(0))
        s = s + add[None]
    p = softmax(s, axis=-1)
    return np.einsum("hqk,khd->qhd", p, vv, dtype=np.float32).astype(np.float32)


def l2_normalize(x: np.ndarray, eps_inside: float | None = 1e-12,
                 clamp_min: float | None = None) -> np.ndarray:
    """Row L2 normalisation in f32.

    ``eps_inside``: ``x / sqrt(sum x^2 + eps)`` (Qwen3 embedder,
    crates/inl-text/src/qwen3/mod.rs:468-469). ``clamp_min``: ``x / max(|x|, c)``
    (F.normalize in the late head, crates/inl-late/src/native.rs:653-661).
    """
    x = x.astype(np.float32, copy=False)
    ss = np.sum(x * x, axis=-1, keepdims=True, dtype=np.float32)
    if clamp_min is not None:
        return (x / np.maximum(np.sqrt(ss), np.float32(clamp_min))).astype(np.float32)
    return (x / np.sqrt(ss + np.float32(eps_inside))).astype(np.float32)


def truncate_and_normalize(v: np.ndarray, dim: int) -> np.ndarray:
    """Matryoshka: keep the first ``dim`` values and renormalise when the norm
    is positive (crates/inl-text/src/native.rs:822-830)."""
    t = v[..., :dim].astype(np.float32)
    n = np.sqrt(np.sum(t * t, axis=-1, keepdims=True, dtype=np.float32))
    return np.where(n > 0, t / np.where(n > 0, n, 1), t).astype(np.float32)


def segments(cu_seqlens: np.ndarray):
    """Yield (start, end) of every packed text."""
    for i in range(len(cu_seqlens) - 1):
        yield int(cu_seqlens[i]), int(cu_seqlens[i + 1])
