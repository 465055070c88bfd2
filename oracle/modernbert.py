"""ModernBERT masked-LM encoder + SPLADE pooling on the CPU (numpy f32):
TEST INFRASTRUCTURE ONLY.

Restates crates/inl-sparse/src/modernbert.rs (config 2 and the reference's
tiny_splade golden fixture) over packed variable-length inputs:

* tower (ModernBertMlm::hidden_states, :621-654): token embedding, LayerNorm
  without bias, layers of ``h += Attn(LN?(h))`` (no norm before layer 0's
  attention, :488-492) and ``h += Wo(gelu_erf(Wi_in h) * Wi_gate h)`` (:406-430),
  final LayerNorm. Layer ``i`` is global iff ``i % global_attn_every_n_layers
  == 0`` (:147-149); local layers mask keys with ``|q - k| > local_attention/2``
  (:594-617). RoPE per layer type with its own theta, half-split (:226-270).
* head (:657-662): ``decoder(LN(gelu_erf(dense(h))))`` with the decoder tied to
  the token embeddings and its bias deferred.
* pooling (SpladePooling::pool_states / finish / fold, :806-907): over the
  text's speaking positions (tokens whose id is not a prefix id),
  ``m_v = max_t logit[t, v]``; ``w_v = ln(1 + relu(m_v + b_v - shift)) * open_v``
  (a text with no speaking position pools to 0); optional max-fold onto
  canonical term ids.
"""
from __future__ import annotations

import numpy as np

from .common import apply_rope, attend_text, gelu_erf, layer_norm, rope_table, segments


def config_values(cfg: dict) -> dict:
    """The fields ModernBertConfig reads (crates/inl-sparse/src/modernbert.rs:28-166)."""
    H = int(cfg["hidden_size"])
    heads = int(cfg["num_attention_heads"])
    eps = cfg.get("norm_eps", cfg.get("layer_norm_eps", 1e-5))
    rp = cfg.get("rope_parameters")
    if rp:
        g_theta = float(rp["full_attention"]["rope_theta"])
        l_theta = float(rp["sliding_attention"]["rope_theta"])
    else:
        g_theta = float(cfg["global_rope_theta"])
        l_theta = float(cfg["local_rope_theta"])
    return {
        "H": H, "I": int(cfg["intermediate_size"]), "heads": heads, "d": H // heads,
        "layers": int(cfg["num_hidden_layers"]), "V": int(cfg["vocab_size"]), "eps": float(eps),
        "half_window": int(cfg.get("local_attention", 128)) // 2,
        "global_every": int(cfg.get("global_attn_every_n_layers", 3)),
        "g_theta": g_theta, "l_theta": l_theta,
    }


def _w(weights: dict, name: str) -> np.ndarray:
    return np.asarray(weights[name], dtype=np.float32)


def hidden_states(weights: dict, cfg: dict, ids: np.ndarray, cu_seqlens: np.ndarray) -> np.ndarray:
    """Final hidden state after final_norm, [T, H]."""
    c = config_values(cfg)
    ids = np.asarray(ids, dtype=np.int64)
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    H, I, heads, d, eps = c["H"], c["I"], c["heads"], c["d"], c["eps"]
    T = len(ids)
    max_len = int(np.max(np.diff(cu))) if len(cu) > 1 else 1
    g_cos, g_sin = rope_table(d, c["g_theta"], max(max_len, 1))
    l_cos, l_sin = rope_table(d, c["l_theta"], max(max_len, 1))
    h = layer_norm(_w(weights, "model.embeddings.tok_embeddings.weight")[ids],
                   _w(weights, "model.embeddings.norm.weight"), None, eps)
    for i in range(c["layers"]):
        p = f"model.layers.{i}."
        glob = i % c["global_every"] == 0
        x = h if i == 0 else layer_norm(h, _w(weights, p + "attn_norm.weight"), None, eps)
        qkv = x @ _w(weights, p + "attn.Wqkv.weight").T
        q = qkv[:, :H].reshape(T, heads, d)
        k = qkv[:, H:2 * H].reshape(T, heads, d)
        v = qkv[:, 2 * H:].reshape(T, heads, d)
        cos, sin = (g_cos, g_sin) if glob else (l_cos, l_sin)
        out = np.empty((T, heads, d), dtype=np.float32)
        for s, e in segments(cu):
            L = e - s
            if L == 0:
                continue
            qs = apply_rope(q[s:e], cos[:L], sin[:L])
            ks = apply_rope(k[s:e], cos[:L], sin[:L])
            out[s:e] = attend_text(qs, ks, v[s:e], d ** -0.5, causal=False,
                                   window=None if glob else c["half_window"])
        h = (h + out.reshape(T, H) @ _w(weights, p + "attn.Wo.weight").T).astype(np.float32)
        x = layer_norm(h, _w(weights, p + "mlp_norm.weight"), None, eps)
        wi = x @ _w(weights, p + "mlp.Wi.weight").T
        h = (h + (gelu_erf(wi[:, :I]) * wi[:, I:]) @ _w(weights, p + "mlp.Wo.weight").T).astype(np.float32)
    return layer_norm(h, _w(weights, "model.final_norm.weight"), None, eps)


def mlm_logits(weights: dict, cfg: dict, states: np.ndarray) -> np.ndarray:
    """Bias-free decoder logits of packed states [t, H] -> [t, V] (project, :657-662)."""
    eps = config_values(cfg)["eps"]
    x = gelu_erf(states @ _w(weights, "head.dense.weight").T)
    x = layer_norm(x, _w(weights, "head.norm.weight"), None, eps)
    return (x @ _w(weights, "model.embeddings.tok_embeddings.weight").T).astype(np.float32)


def pooling_dimension(pooling: dict, vocab: int) -> int:
    """max(canonical_ids) + 1, else the vocabulary (SpladePooling::dimension, :775-781)."""
    canon = pooling.get("canonical_ids")
    return int(max(canon)) + 1 if canon else vocab


def splade(weights: dict, cfg: dict, pooling: dict, ids: np.ndarray, cu_seqlens: np.ndarray,
           block: int = 128) -> np.ndarray:
    """Dense SPLADE rows [n, dimension] (ModernBertMlm::splade, :671-691)."""
    c = config_values(cfg)
    V = c["V"]
    ids = np.asarray(ids, dtype=np.int64)
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    states = hidden_states(weights, cfg, ids, cu)
    prefix = set(int(x) for x in pooling.get("prefix_token_ids", []))
    n = len(cu) - 1
    best = np.full((n, V), -np.inf, dtype=np.float32)
    for i, (s, e) in enumerate(segments(cu)):
        speak = [t for t in range(s, e) if int(ids[t]) not in prefix]
        for b in range(0, len(speak), block):  # the reference's LOGIT_TOKENS blocks; max is exact
            rows = speak[b:b + block]
            logits = mlm_logits(weights, cfg, states[rows])
            best[i] = np.maximum(best[i], logits.max(axis=0))
    bias = np.asarray(weights.get("decoder.bias", np.zeros(V)), dtype=np.float32)
    open_ = np.ones(V, dtype=np.float32)
    for v in pooling.get("masked_vocab_ids", []):
        open_[int(v)] = 0.0
    shift = np.float32(pooling.get("logit_shift", 0.0))
    # finish (:879-885): relu before the mask so -inf never meets a zero
    w = np.log(np.float32(1.0) + np.maximum(best + bias - shift, 0.0) * open_).astype(np.float32)
    canon = pooling.get("canonical_ids")
    if not canon:
        return w
    dim = pooling_dimension(pooling, V)
    out = np.zeros((n, dim), dtype=np.float32)
    for v, term in enumerate(canon):  # fold (:888-907): max per canonical term
        out[:, term] = np.maximum(out[:, term], w[:, v])
    return out


def sparse(dense_row: np.ndarray) -> tuple[list[int], list[float]]:
    """SparseVector::from_pairs (crates/inl-sparse/src/lib.rs:51-62): indices of
    weights > 0 (NaN dropped), sorted, with their values."""
    idx = [int(i) for i in np.nonzero(dense_row > 0)[0]]
    return idx, [float(dense_row[i]) for i in idx]
