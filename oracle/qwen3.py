"""Qwen3 encoder forward on the CPU (numpy f32): TEST INFRASTRUCTURE ONLY.

Restates crates/inl-text/src/qwen3/mod.rs (the Qwen3 embedder, configs 1 and 5)
over packed variable-length inputs, and composes it with the late-interaction
head of crates/inl-late/src/native.rs:631-683 (config 3: bidirectional tower,
final norm on every token, 1024->128 projection, F.normalize).

Packing note: the reference left-pads a batch and masks padded keys with -1e4
(crates/inl-core/src/attention.rs:170-199); RoPE positions then start at the
pad length, a shift attention is invariant to (the reference pins this with
its padding-invariance test, crates/inl-text/src/qwen3/mod.rs:646-669). The
packed form used here gives every text positions 0..L-1 and attends only
within the text, which is the same function.

Parity: unpinned by golden vectors (partial). The reference's only Qwen3
golden (crates/inl-text/tests/fixtures/qwen3embedding/golden_real.json) needs
the real checkpoint, which is absent. tests/test_oracle_qwen3.py checks this
restatement against the reference's own unit-test invariants and against
transformers' Qwen3Model on the same random weights (a second opinion, not
the reference).
"""
from __future__ import annotations

import numpy as np

from .common import apply_rope, attend_text, l2_normalize, rms_norm, rope_table, segments, silu


def _w(weights: dict, name: str) -> np.ndarray:
    return np.asarray(weights[name], dtype=np.float32)


def layer_forward(weights: dict, cfg: dict, i: int, h: np.ndarray, cu_seqlens: np.ndarray,
                  cos: np.ndarray, sin: np.ndarray, causal: bool) -> np.ndarray:
    """One DecoderLayer: ``h += Attn(RMSNorm(h)); h += MLP(RMSNorm(h))``.

    crates/inl-text/src/qwen3/mod.rs:282-297 (layer), :227-254 (attention:
    q/k/v projections, per-head q/k RMSNorm, RoPE, GQA, o projection),
    :110-116 (SwiGLU MLP).
    """
    p = f"layers.{i}."
    eps = float(cfg["rms_norm_eps"])
    hq, hkv = int(cfg["num_attention_heads"]), int(cfg["num_key_value_heads"])
    d = int(cfg.get("head_dim") or cfg["hidden_size"] // hq)
    T = h.shape[0]
    x = rms_norm(h, _w(weights, p + "input_layernorm.weight"), eps)
    q = (x @ _w(weights, p + "self_attn.q_proj.weight").T).reshape(T, hq, d)
    k = (x @ _w(weights, p + "self_attn.k_proj.weight").T).reshape(T, hkv, d)
    v = (x @ _w(weights, p + "self_attn.v_proj.weight").T).reshape(T, hkv, d)
    if cfg.get("attention_bias"):
        q = q + _w(weights, p + "self_attn.q_proj.bias").reshape(hq, d)
        k = k + _w(weights, p + "self_attn.k_proj.bias").reshape(hkv, d)
        v = v + _w(weights, p + "self_attn.v_proj.bias").reshape(hkv, d)
    q = rms_norm(q, _w(weights, p + "self_attn.q_norm.weight"), eps)
    k = rms_norm(k, _w(weights, p + "self_attn.k_norm.weight"), eps)
    out = np.empty((T, hq, d), dtype=np.float32)
    scale = d ** -0.5
    for s, e in segments(cu_seqlens):
        L = e - s
        if L == 0:
            continue
        qs = apply_rope(q[s:e], cos[:L], sin[:L])
        ks = apply_rope(k[s:e], cos[:L], sin[:L])
        out[s:e] = attend_text(qs, ks, v[s:e], scale, causal=causal)
    o = out.reshape(T, hq * d) @ _w(weights, p + "self_attn.o_proj.weight").T
    if cfg.get("attention_bias"):
        o = o + _w(weights, p + "self_attn.o_proj.bias")
    h = (h + o).astype(np.float32)
    x = rms_norm(h, _w(weights, p + "post_attention_layernorm.weight"), eps)
    g = x @ _w(weights, p + "mlp.gate_proj.weight").T
    u = x @ _w(weights, p + "mlp.up_proj.weight").T
    m = (silu(g) * u) @ _w(weights, p + "mlp.down_proj.weight").T
    return (h + m).astype(np.float32)


def hidden_states(weights: dict, cfg: dict, ids: np.ndarray, cu_seqlens: np.ndarray,
                  causal: bool = True) -> np.ndarray:
    """Embedding + every layer, before the final norm: [T, H].

    crates/inl-text/src/qwen3/mod.rs:339-358 (forward_last without the final
    narrow/norm).
    """
    ids = np.asarray(ids, dtype=np.int64)
    cu_seqlens = np.asarray(cu_seqlens, dtype=np.int64)
    hq = int(cfg["num_attention_heads"])
    d = int(cfg.get("head_dim") or cfg["hidden_size"] // hq)
    max_len = int(np.max(np.diff(cu_seqlens))) if len(cu_seqlens) > 1 else 0
    cos, sin = rope_table(d, float(cfg["rope_theta"]), max(max_len, 1))
    h = _w(weights, "embed_tokens.weight")[ids]
    for i in range(int(cfg["num_hidden_layers"])):
        h = layer_forward(weights, cfg, i, h, cu_seqlens, cos, sin, causal)
    return h


def embed_last(weights: dict, cfg: dict, ids: np.ndarray, cu_seqlens: np.ndarray) -> np.ndarray:
    """Dense embeddings [n, H]: final RMSNorm of each text's last token, then
    ``x / sqrt(sum x^2 + 1e-12)`` in f32.

    crates/inl-text/src/qwen3/mod.rs:339-358 (last position, final norm) and
    :438-470 (f32 L2).
    """
    cu_seqlens = np.asarray(cu_seqlens, dtype=np.int64)
    h = hidden_states(weights, cfg, ids, cu_seqlens, causal=True)
    last = h[cu_seqlens[1:] - 1]
    pooled = rms_norm(last, _w(weights, "norm.weight"), float(cfg["rms_norm_eps"]))
    return l2_normalize(pooled, eps_inside=1e-12)


def encode_late(weights: dict, cfg: dict, projection: np.ndarray, ids: np.ndarray,
                cu_seqlens: np.ndarray, bias: np.ndarray | None = None) -> np.ndarray:
    """Per-token late-interaction vectors [T, out]: bidirectional tower, final
    RMSNorm on every token, f32 projection, F.normalize (clamp 1e-12).

    Tower mask: padding only, no causal part (the non-causal branch of
    crates/inl-late/src/qwen3_5.rs:914-927). Head:
    crates/inl-late/src/native.rs:646-661. ``projection`` is the Dense
    ``linear.weight`` [out, H].
    """
    h = hidden_states(weights, cfg, ids, cu_seqlens, causal=False)
    x = rms_norm(h, _w(weights, "norm.weight"), float(cfg["rms_norm_eps"]))
    y = x @ np.asarray(projection, dtype=np.float32).T
    if bias is not None:
        y = y + bias
    return l2_normalize(y, clamp_min=1e-12)
