"""EmbeddingGemma text tower on the CPU (numpy f32): TEST INFRASTRUCTURE ONLY.

Restates crates/inl-text/src/gemma2.rs over packed variable-length inputs:

* embeddings ``embed_tokens[ids] * sqrt(H)`` (:575-587, :606-608);
* optional per-layer embeddings (PLE, :279-283, :622-630):
  ``RMSNorm(reshape(E W_ple^T * H^-1/2, [T, layers, ple]))``;
* per layer (:473-494): ``h += postN(Attn(inN(h)))``,
  ``h += postFF(down(gelu_tanh(gate(preFF h)) * up(preFF h)))``, then, with PLE,
  ``h = (h + postPLE(proj(gelu_tanh(gate_ple(h)) * ple_i))) * layer_scalar``;
* attention (:381-441): q/k RMSNorm with weight, v RMSNorm without weight,
  half-split RoPE with the layer kind's theta and head shape, UNSCALED scores
  (scale 1), softmax in f32, sliding layers mask ``|q - k| > sliding_window``
  (:499-523, additive -1e9), GQA by head index;
* final RMSNorm, mean over the text's tokens, projection, f32 L2 with 1e-12
  inside the root (:648-661).

``embed`` is the reference's pipeline (projection = ``embedding_projection``),
pinned by the tiny_embeddinggemma2 golden. ``embed_dense_head`` is the
benchmark's config-4 variant: no PLE / layer scalar, the projection replaced by
a dense 768->3072->768 chain, then Matryoshka truncate-and-renormalise
(crates/inl-text/src/native.rs:822-830).
"""
from __future__ import annotations

import math

import numpy as np

from .common import (apply_rope, attend_text, gelu_tanh, l2_normalize, rms_norm, rope_table, segments,
                     truncate_and_normalize)

MASKED = np.float32(-1e9)  # crates/inl-text/src/gemma2.rs:41


def text_config(cfg: dict) -> dict:
    return cfg["text_config"] if "text_config" in cfg else cfg


def layer_shape(tc: dict, index: int) -> tuple[str, int, int]:
    """(kind, head_dim, kv_heads) with per_layer_config overrides (:186-204)."""
    kinds = tc.get("layer_types")
    if kinds:
        kind = kinds[index]
    else:  # full attention every `full_attention_every_n_layers`-th layer (idx % n == n - 1)
        n = int(tc.get("full_attention_every_n_layers", 6))
        kind = "full_attention" if index % n == n - 1 else "sliding_attention"
    over = {}
    for k, v in (tc.get("per_layer_config") or {}).items():
        if int(k) == index:
            over = v
    return kind, int(over.get("head_dim") or tc["head_dim"]), int(over.get("num_key_value_heads")
                                                                     or tc["num_key_value_heads"])


def _w(weights: dict, name: str) -> np.ndarray:
    return np.asarray(weights[name], dtype=np.float32)


def _thetas(tc: dict) -> tuple[float, float]:
    rp = tc.get("rope_parameters")
    if rp:
        return float(rp["full_attention"]["rope_theta"]), float(rp["sliding_attention"]["rope_theta"])
    return float(tc.get("rope_theta", 1e6)), float(tc.get("rope_local_base_freq", 1e4))


def final_hidden(weights: dict, cfg: dict, ids, cu_seqlens, prefix: str = "language_model.",
                 embed_scale: float | None = None) -> np.ndarray:
    """Final-normed hidden states [T, H]."""
    tc = text_config(cfg)
    ids = np.asarray(ids, dtype=np.int64)
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    H, layers, heads = int(tc["hidden_size"]), int(tc["num_hidden_layers"]), int(tc["num_attention_heads"])
    eps = float(tc["rms_norm_eps"])
    window = int(tc["sliding_window"])
    T = len(ids)
    w = lambda n: _w(weights, prefix + n)  # noqa: E731
    scale = np.float32(math.sqrt(H) if embed_scale is None else embed_scale)
    h = w("embed_tokens.weight")[ids] * scale
    ple_dim = int(tc.get("hidden_size_per_layer_input") or 0)
    use_ple = ple_dim > 0 and (prefix + "ple.per_layer_model_projection.weight") in weights
    if use_ple:
        per = (h @ w("ple.per_layer_model_projection.weight").T) * np.float32(H ** -0.5)
        per = rms_norm(per.reshape(T, layers, ple_dim), w("ple.per_layer_projection_norm.weight"), eps)
    max_len = int(np.max(np.diff(cu))) if len(cu) > 1 else 1
    full_theta, slide_theta = _thetas(tc)
    tables = {}
    for i in range(layers):
        p = f"layers.{i}."
        kind, d, kvh = layer_shape(tc, i)
        key = (kind, d)
        if key not in tables:
            tables[key] = rope_table(d, full_theta if kind == "full_attention" else slide_theta, max(max_len, 1))
        cos, sin = tables[key]
        x = rms_norm(h, w(p + "input_layernorm.weight"), eps)
        q = rms_norm((x @ w(p + "self_attn.q_proj.weight").T).reshape(T, heads, d), w(p + "self_attn.q_norm.weight"), eps)
        k = rms_norm((x @ w(p + "self_attn.k_proj.weight").T).reshape(T, kvh, d), w(p + "self_attn.k_norm.weight"), eps)
        v = rms_norm((x @ w(p + "self_attn.v_proj.weight").T).reshape(T, kvh, d), None, eps)
        out = np.empty((T, heads, d), dtype=np.float32)
        for s, e in segments(cu):
            L = e - s
            if L == 0:
                continue
            out[s:e] = attend_text(apply_rope(q[s:e], cos[:L], sin[:L]), apply_rope(k[s:e], cos[:L], sin[:L]),
                                   v[s:e], 1.0, causal=False,
                                   window=None if kind == "full_attention" else window, mask_value=MASKED)
        a = out.reshape(T, heads * d) @ w(p + "self_attn.o_proj.weight").T
        h = (h + rms_norm(a, w(p + "post_attention_layernorm.weight"), eps)).astype(np.float32)
        x = rms_norm(h, w(p + "pre_feedforward_layernorm.weight"), eps)
        m = (gelu_tanh(x @ w(p + "mlp.gate_proj.weight").T) * (x @ w(p + "mlp.up_proj.weight").T)) \
            @ w(p + "mlp.down_proj.weight").T
        h = (h + rms_norm(m, w(p + "post_feedforward_layernorm.weight"), eps)).astype(np.float32)
        if use_ple:
            g = gelu_tanh(h @ w(p + "ple_block.per_layer_input_gate.weight").T) * per[:, i, :]
            g = rms_norm(g @ w(p + "ple_block.per_layer_projection.weight").T,
                         w(p + "ple_block.post_per_layer_input_norm.weight"), eps)
            h = ((h + g) * w(p + "layer_scalar")).astype(np.float32)
    return rms_norm(h, w("norm.weight"), eps)


def mean_pool(h: np.ndarray, cu_seqlens) -> np.ndarray:
    """Mean over each text's tokens (the masked mean of :648-656)."""
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    out = np.zeros((len(cu) - 1, h.shape[1]), dtype=np.float32)
    for i, (s, e) in enumerate(segments(cu)):
        if e > s:
            out[i] = h[s:e].mean(axis=0, dtype=np.float32)
    return out


def embed(weights: dict, cfg: dict, ids, cu_seqlens, prefix: str = "language_model.") -> np.ndarray:
    """The reference pipeline: mean pool, embedding_projection, f32 L2 (:622-662)."""
    h = final_hidden(weights, cfg, ids, cu_seqlens, prefix)
    pooled = mean_pool(h, cu_seqlens)
    proj = pooled @ _w(weights, prefix + "embedding_projection.weight").T
    return l2_normalize(proj, eps_inside=1e-12)


def embed_dense_head(weights: dict, cfg: dict, dense: list[np.ndarray], ids, cu_seqlens, out_dim: int = 0,
                     prefix: str = "") -> np.ndarray:
    """Config 4: mean pool -> dense chain (no activation) -> L2 -> Matryoshka."""
    h = final_hidden(weights, cfg, ids, cu_seqlens, prefix)
    x = mean_pool(h, cu_seqlens)
    for wd in dense:
        x = x @ np.asarray(wd, dtype=np.float32).T
    x = l2_normalize(x, eps_inside=1e-12)
    return truncate_and_normalize(x, out_dim) if out_dim else x
